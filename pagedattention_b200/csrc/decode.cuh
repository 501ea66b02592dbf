// Paged-attention decode kernels for sm_100a.
//
// Reference path (lashhw/pagedattention):
//   planner        src/kernel_triton.py:206-243  (host, with a device sync)
//   split kernel   src/kernel_triton.py:8-117    (one program per chunk x q head)
//   reduce kernel  src/kernel_triton.py:120-174  (log-sum-exp merge of chunks)
//   numerics       src/kernel_eager.py:29-56     (softmax(q K^T * scale) V)
//
// Design here:
//   plan_kernel    one CTA.  Clamps every sequence length, prefix-sums the
//                  page counts of all (sequence, kv head) pairs ("heads" below)
//                  into `cum`, and gives every warp of the decode grid its
//                  first head; lists the heads of length 0.
//   decode_kernel  persistent.  The concatenation of all heads' pages is cut
//                  into W equal contiguous ranges, one per warp (W = every
//                  resident warp on the device), so the load is balanced to a
//                  page whatever the length mix.  The last `m` chunks of `K`
//                  pages of every range are claimed at run time (one 64-bit
//                  atomic word per warp): the owner takes them from the front,
//                  warps that ran out of work steal them from the back, which
//                  evens out the speed differences between warps (SM position,
//                  HBM channel mix) that a static split leaves as a tail.
//                  Each warp streams its pages
//                  through a private ring of shared-memory stages filled by
//                  tensor-map bulk copies (TMA, 128-byte swizzle, mbarrier
//                  completion), computes S^T = K Q^T and O^T += V^T P^T with
//                  mma.sync m16n8k16 (tokens are the M dimension, the G query
//                  heads of one kv head the N dimension, so one K/V read
//                  serves the whole group) and keeps an online softmax in
//                  registers.  A head lying wholly in one segment (the static
//                  prefix or one chunk of a range) is written directly; a
//                  head split over several segments has each segment write a
//                  partial (max, sum, acc) with plain stores.  Segments,
//                  partials and merge order are fixed by the page counts
//                  alone, so results do not depend on which warp ran which
//                  chunk.
//   reduce kernels merge the split heads' partials after the decode grid
//                  (the reduce kernel of the reference): one warp per head
//                  (lanes over its G x D outputs) or per (head, query head)
//                  row for large groups, or, when heads have many partials,
//                  one CTA per row whose warps split the partials.
//
// Launch chain (programmatic dependent launch): every kernel lets the next
// one start before it ends, and every kernel writes nothing before its
// dependency wait — until then it only reads inputs and its own shared
// memory.  So the next call's planner and decode grid start while this
// call's decode grid drains and its reduce runs: the planner plans, the
// decode CTAs (when the call allows an early start) prefix-sum the lengths,
// take over SMs as this call's CTAs leave and stream their first pages; the
// first write of a call (planner: its plan; decode: an output, a partial
// state, a claim, a status bit) waits for the previous call to finish.
//
// Shared-memory stage layout (per warp, per ring slot), ST tokens:
//   K: [D/64 planes][ST rows][128 bytes], then V with the same shape.
//   A plane holds 64 consecutive head-dim elements of every token; its
//   128-byte rows are 128B-swizzled by the TMA unit (16-byte chunk c of row r
//   is stored at chunk c ^ (r % 8)), which makes every ldmatrix below
//   bank-conflict free.
#pragma once

#include <type_traits>

#include "ptx.cuh"

namespace pab {

constexpr int kMaxDepth = 8;                      // ring slots per warp (max)
constexpr int kMaxWarpsPerCta = 8;                // keeps 255 registers/thread
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per pipeline wait
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kStatusBadPage = 0x1u;
constexpr uint32_t kStatusClamp = 0x2u;
constexpr uint32_t kStatusNegative = 0x4u;
constexpr uint32_t kStatusTimeout = 0x8u;
constexpr int kMetaBytesPerSlot = 32;  // two int4 per ring slot
constexpr int kCoreMaxG = 4;           // largest query group of the CUDA-core path
// Early start of the decode grid: calls with at most this many (sequence,
// kv head) pairs keep their page-count prefix in shared memory.
constexpr int kEarlyMaxHeads = 1024;
constexpr int kEarlyBytes = (2 * kEarlyMaxHeads + 1 + 32) * 4;  // cum, lengths, warp sums

// tcgen05 path (query groups of up to 32 heads, D 64, 64-token stages): a
// unit of two warps per ring; tensor-memory columns per unit (two score
// buffers of 32 columns, the 64-column output accumulator); bytes of one
// 64-row x 128-byte operand tile (queries, or probabilities).
constexpr int kTcUnitCols = 128;
constexpr int kTcTileBytes = 64 * 128;
// Offsets, from the start of the tail (after the paired layout's stage
// mbarriers, stage records and slot-free mbarriers), of the tcgen05 path's
// per-unit mbarriers and of the tensor-memory base address.
constexpr int kTcBarsPerUnit = 6;
__host__ __device__ constexpr int tc_bars_offset(int upc) {
  return upc * kMaxDepth * (8 + kMetaBytesPerSlot) + upc * kMaxDepth * 8;
}
__host__ __device__ constexpr int tc_slot_offset(int upc) {
  return tc_bars_offset(upc) + upc * kTcBarsPerUnit * 8;
}

// Per-warp shared memory of the CUDA-core path: the query group in fp32.
__host__ __device__ constexpr int core_q_bytes(bool core, int D) {
  return core ? kCoreMaxG * D * 4 : 0;
}

// Arguments of a KV append (kv_append_kernel, or the planner when a decode
// call appends its step's token first).
struct AppendParams {
  uint32_t* k_cache;
  uint32_t* v_cache;
  const uint32_t* k_new;
  const uint32_t* v_new;
  int32_t* lens;
  const int32_t* bt;
  uint32_t* status;
  int32_t B, Hkv, D, bs, maxb, head_in_page;  // head_in_page: NHD cache (Hkv rows per token)
  int64_t num_pages;
  int64_t n_sb, n_sh, l_sb, l_sh, bt_sb, bt_sh, bt_si;
  int32_t bt_mul, bt_add, increment;
  int32_t vec16;  // rows copied as 16-byte units (new rows and caches 16-byte aligned)
};

constexpr uint32_t kStatusAppendFull = 0x10u;

struct DecodeParams {
  void* out;
  const void* q;
  const int32_t* lens;
  const int32_t* bt;
  int64_t q_sb, q_sh, o_sb, o_sh, l_sb, l_sh, bt_sb, bt_sh, bt_si;
  int32_t bt_mul, bt_add;
  int32_t B, Hkv, G, D, bs, maxb;
  int64_t num_pages;
  int32_t head_in_map;  // NHD layout: kv head is the tensor map's y coordinate
  float scale_log2;     // softmax_scale * log2(e)
  int32_t total_warps;  // W
  int32_t depth;        // ring slots per warp
  // workspace
  int32_t* cum;       // [n_heads + 1] exclusive prefix of page counts
  int32_t* wstart;    // [W] first head of each warp's page range
  uint32_t* status;   // [1] PAB200_STATUS_* bits
  int32_t* weff;      // [1] warps in use: min(total_warps, total pages)
  // [4] dynamic tail, written by the planner: m (tail chunks per warp), K
  // (pages per chunk), chunks left to claim, thief cursor
  int32_t* steal;
  unsigned long long* claims;  // [W] claim words: low 32 bits front, high back
  // [n_heads] first segment and segment count of every head (0 if empty),
  // in two halves: .xy for parity 0, .zw for parity 1, used by alternate
  // calls.
  int4* hseg;
  uint32_t* parity;            // which half of hseg the current call uses
  int32_t* n_empty;            // [1] heads of length 0 in this call
  int32_t* empty;              // [n_heads] their indices (zeroed by the decode grid)
  int32_t steal_m_max;         // tail chunks per warp the workspace holds
  int32_t steal_pps;           // pages per ring stage (ST / block_size)
  int32_t steal_min_stages;    // smallest tail chunk, in ring stages
  // Early start (no append, n_heads <= kEarlyMaxHeads, single-warp rings
  // or the tcgen05 path):
  // the decode grid plans its own ranges and issues its first copies while
  // the planner runs; it waits for the planner only before touching shared
  // state (claims, outputs, status, empty heads).
  int32_t early;
  // [(n_heads + W * (steal_m_max + 1)) * slot_floats] partial states, one
  // per (head, segment) pair; slot layout: acc [G][D], m [G], l [G]
  float* part;
  int32_t slot_floats;
  // cross-device state output (optional)
  float* state_o;
  float* state_lse;
  // optional: append each (sequence, kv head)'s new token before planning
  int32_t append;
  AppendParams app;
};

// Dynamic tail of a call with `total` pages over W warp ranges: about a
// quarter of every range, in at most m_max chunks of whole stages (`pps`
// pages each), each at least `min_stages` stages long; none when the tail
// is shorter than that.  (A claim costs a few dependent L2 atomics, as long
// as streaming a stage or two: short chunks cost more than the balance they
// buy.)  Sets *m (chunks per range) and *k (pages per chunk).
__host__ __device__ __forceinline__ void tail_chunks(int64_t total, int W, int m_max, int pps,
                                                     int min_stages, int* m, int* k) {
  *m = 0;
  *k = 0;
  if (W <= 1 || m_max <= 0) return;
  const int ppw = static_cast<int>(total / W);
  const int tail = ppw / 4;
  const int kmin = pps * (min_stages > 1 ? min_stages : 1);
  if (tail < kmin) return;
  const int each = (tail + m_max - 1) / m_max;
  int kk = (each + pps - 1) / pps * pps;
  if (kk < kmin) kk = kmin;
  int mm = tail / kk;
  if (mm > m_max) mm = m_max;
  *m = mm;
  *k = mm == 0 ? 0 : kk;
}

// The warp that owns global page P (0 <= P < T).  Warp w owns pages
// [floor(w*T/W), floor((w+1)*T/W)).
__device__ __forceinline__ int warp_of_page(int64_t P, int64_t T, int W) {
  return static_cast<int>(((P + 1) * W - 1) / T);
}

// Segment of global page P: warp w's range is a static prefix (segment
// w*(m+1)) followed by m chunks of K pages (segments w*(m+1) + 1 .. m).  The
// pages of a head that fall in one segment form one unit of work and one
// partial state (unless the head lies wholly in the segment); heads and
// segments are both ordered by page, so slot head + segment is unique and a
// head's partials fill slots [head + seg(first page), head + seg(last page)].
// Which warp computes a segment is decided at run time, but the segments,
// their partial states and the merge order are not: results do not depend
// on the schedule.
__device__ __forceinline__ int segment_of_page(int P, int T, int W, int m, int K) {
  const int w = warp_of_page(P, T, W);
  if (m == 0) return w;
  const int t = static_cast<int>(static_cast<int64_t>(w + 1) * T / W) - m * K;
  return w * (m + 1) + (P < t ? 0 : 1 + (P - t) / K);
}

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float x) {
  return __float2half_rn(x);
}

// --------------------------------------------------------------------------
// KV append inside the planner (1024 threads).  Row r = (sequence r / Hkv,
// kv head r % Hkv): its page and destination row at the current length L, or
// -1 when there is no slot (L past max_blocks * bs) or the page id is out of
// range (the status bit is raised by the caller's first pass).
__device__ __forceinline__ int64_t append_row(const AppendParams& a, int s, int h, int L,
                                              uint32_t* flags) {
  if (L < 0) return -1;
  if (L / a.bs >= a.maxb) {
    if (flags) *flags |= kStatusAppendFull;
    return -1;
  }
  const int64_t pid =
      static_cast<int64_t>(a.bt[s * a.bt_sb + h * a.bt_sh + static_cast<int64_t>(L / a.bs) * a.bt_si]) *
          a.bt_mul + static_cast<int64_t>(h) * a.bt_add;
  if (pid < 0 || pid >= a.num_pages) {
    if (flags) *flags |= kStatusBadPage;
    return -1;
  }
  return (pid * a.bs + L % a.bs) * (a.head_in_page ? a.Hkv : 1) + (a.head_in_page ? h : 0);
}

// Pass 1, in chunks of 1024 rows: thread t resolves row t's destination
// (one round of length and block-table loads), then all 1024 threads copy
// the chunk's K and V rows in 16-byte units (4-byte words when unaligned).
// Lengths are not written here, so every row reads its length before any
// changes.
__device__ __forceinline__ void planner_append_rows(const AppendParams& a, int tid) {
  __shared__ int64_t dst[1024];
  __shared__ int64_t src_sm[1024];
  const int rows = a.B * a.Hkv;
  const int unit_words = a.vec16 ? 4 : 1;
  const int units = a.D / 2 / unit_words;  // per row
  uint32_t flags = 0;
  for (int c0 = 0; c0 < rows; c0 += 1024) {
    const int r = c0 + tid;
    if (r < rows) {
      const int s = r / a.Hkv, h = r - s * a.Hkv;
      const int L = a.lens[s * a.l_sb + h * a.l_sh];
      dst[tid] = append_row(a, s, h, L, &flags);
      src_sm[tid] = (s * a.n_sb + static_cast<int64_t>(h) * a.n_sh) / 2;
    }
    __syncthreads();
    const int n = min(1024, rows - c0);
    for (int u = tid; u < n * units; u += 1024) {
      const int rr = u / units, part = u - rr * units;
      const int64_t row = dst[rr];
      if (row < 0) continue;
      const int64_t so = src_sm[rr] + part * unit_words;
      const int64_t doff = row * (a.D / 2) + part * unit_words;
      if (a.vec16) {
        *reinterpret_cast<uint4*>(a.k_cache + doff) = *reinterpret_cast<const uint4*>(a.k_new + so);
        *reinterpret_cast<uint4*>(a.v_cache + doff) = *reinterpret_cast<const uint4*>(a.v_new + so);
      } else {
        a.k_cache[doff] = a.k_new[so];
        a.v_cache[doff] = a.v_new[so];
      }
    }
    __syncthreads();  // dst / src_sm are reused by the next chunk
  }
  if (flags && a.status) atomicOr(a.status, flags);
}

// Pass 2 (after a CTA barrier, so every row read its length first): each
// written row's length moves to L + 1; a length shared by a sequence's heads
// moves once, if every head's token was written.
__device__ __forceinline__ void planner_append_lengths(const AppendParams& a, int tid) {
  if (!a.increment) return;
  if (a.l_sh != 0) {
    for (int r = tid; r < a.B * a.Hkv; r += 1024) {
      const int s = r / a.Hkv, h = r - s * a.Hkv;
      int32_t* lp = a.lens + s * a.l_sb + h * a.l_sh;
      const int L = *lp;
      if (append_row(a, s, h, L, nullptr) >= 0) *lp = L + 1;
    }
  } else {
    for (int s = tid; s < a.B; s += 1024) {
      int32_t* lp = a.lens + s * a.l_sb;
      const int L = *lp;
      bool ok = true;
      for (int h = 0; h < a.Hkv; ++h) ok &= append_row(a, s, h, L, nullptr) >= 0;
      if (ok) *lp = L + 1;
    }
  }
}

// --------------------------------------------------------------------------
// Planner: one CTA of 1024 threads.
template <typename T, bool APPEND>
__global__ void __launch_bounds__(1024) plan_kernel(const DecodeParams p) {
  __shared__ int32_t warp_tot[32];
  __shared__ uint32_t par_sm;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_heads = p.B * p.Hkv;
  const int cap = p.maxb * p.bs;
  // This kernel may start while the previous call's kernels on the stream
  // still run (programmatic dependent launch: the previous reduce kernel
  // lets it start at once), and it lets the decode grid start at once.  Nothing is written before the wait for the
  // previous grid below: until then the kernel only loads the lengths
  // (inputs) and computes the plan, so every workspace write of a call
  // follows the end of the previous call, whatever its shapes.
  grid_launch_dependents();
  // Thread t owns heads [t * per, (t + 1) * per): its page counts are loaded
  // in one round (up to kPer of them kept in registers), summed, and one
  // block-wide exclusive scan of the sums gives every head's first page.
  constexpr int kPer = 8;
  const int per = (n_heads + 1023) / 1024;
  const int h0 = tid * per;
  const int h1 = min(h0 + per, n_heads);
  uint32_t flags = 0;
  auto head_pages = [&](int hd) {
    const int s = hd / p.Hkv, h = hd - s * p.Hkv;
    int L = p.lens[s * p.l_sb + h * p.l_sh];
    if (L < 0) {
      flags |= kStatusNegative;
      L = 0;
    } else if (L > cap) {
      flags |= kStatusClamp;
      L = cap;
    }
    return (L + p.bs - 1) / p.bs;
  };
  if constexpr (APPEND) {
    // The step's new tokens go into the cache first, once the previous
    // call (whose decode read the cache) has finished: every row is
    // written at the current length, then the lengths move.
    grid_dependency_wait();
    if (tid == 0) *p.status = 0u;
    __syncthreads();  // status reset before any append bit is raised
    planner_append_rows(p.app, tid);
    __syncthreads();
    planner_append_lengths(p.app, tid);
    __syncthreads();
  }
  int pg[kPer];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    pg[i] = h0 + i < h1 ? head_pages(h0 + i) : 0;
    sum += pg[i];
  }
  for (int hd = h0 + kPer; hd < h1; ++hd) sum += head_pages(hd);
  // Which half of hseg this call uses: the other half from the one the
  // last finished planner chose (any choice would do — no kernel reads hseg
  // before this call's plan is written — but alternating keeps the halves
  // of consecutive calls apart).
  if (tid == 0) par_sm = (*reinterpret_cast<volatile uint32_t*>(p.parity) ^ 1u) & 1u;
  int x = sum;  // inclusive scan within the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int v = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    warp_tot[lane] = v;
  }
  __syncthreads();
  const int64_t total = warp_tot[31];
  int run = (warp ? warp_tot[warp - 1] : 0) + x - sum;  // first page of head h0
  // With more warps than pages some warps would own no page and the span
  // count of a head (warp_of_page(last) - warp_of_page(first) + 1) would
  // include them; capping W at the page count gives every warp >= 1 page.
  const int W = static_cast<int>(total < p.total_warps ? total : p.total_warps);
  // Dynamic tail chunks of every warp range (tail_chunks).
  int sm_m = 0, sm_k = 0;
  tail_chunks(total, W, p.steal_m_max, p.steal_pps, p.steal_min_stages, &sm_m, &sm_k);
  const uint32_t par = par_sm;

  // The previous call's kernels have finished from here on: write the plan.
  if constexpr (!APPEND) grid_dependency_wait();
  if (tid == 0) {
    if constexpr (!APPEND) *p.status = 0u;
    *p.n_empty = 0;
    *p.parity = par;
    *p.weff = W;
    p.steal[0] = sm_m;
    p.steal[1] = sm_k;
    p.steal[2] = sm_m * W;  // chunks left to claim
    p.steal[3] = 0;         // thief cursor
    p.cum[n_heads] = static_cast<int>(total);
  }
  __syncthreads();  // status and empty count reset before the updates below
  if (flags) atomicOr(p.status, flags);
  if (sm_m > 0)
    for (int w = tid; w < W; w += 1024) p.claims[w] = 0ull;
  // Per head: its first page, the warps whose range starts in it, its
  // segment range, or (empty head) its place in the empty list.
  const int tp = static_cast<int>(total);
  auto place_head = [&](int hd, int pages) {
    const int64_t c0 = run, c1 = run + pages;
    p.cum[hd] = run;
    run += pages;
    if (c1 > c0) {
      // warps whose first page lies in [c0, c1)
      const int64_t wa = (c0 * W + total - 1) / total;
      const int64_t wb = (c1 * W + total - 1) / total;
      for (int64_t w = wa; w < wb; ++w) p.wstart[w] = hd;
      const int v0 = segment_of_page(static_cast<int>(c0), tp, W, sm_m, sm_k);
      reinterpret_cast<int2*>(p.hseg + hd)[par] =
          make_int2(v0, segment_of_page(static_cast<int>(c1) - 1, tp, W, sm_m, sm_k) - v0 + 1);
    } else {
      // Empty head: listed here, its zero output is written by the decode
      // grid, after its own wait for this kernel.
      reinterpret_cast<int2*>(p.hseg + hd)[par] = make_int2(0, 0);
      p.empty[atomicAdd(p.n_empty, 1)] = hd;
    }
  };
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (h0 + i < h1) place_head(h0 + i, pg[i]);
  for (int hd = h0 + kPer; hd < h1; ++hd) place_head(hd, head_pages(hd));
}

// --------------------------------------------------------------------------
// Shared-memory helpers of the CUDA-core path.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Eight 16-bit values (one 16-byte chunk) to fp32.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]);
template <>
__device__ __forceinline__ void unpack8<__nv_bfloat16>(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // bf16 -> fp32 is a 16-bit left shift
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack8<__half>(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// DL consecutive 16-bit values at shared address `addr` to fp32 (DL = 2 or 4).
template <typename T, int DL>
__device__ __forceinline__ void load_row_part(uint32_t addr, float (&f)[DL]) {
  float t[8];
  if constexpr (DL == 4) {
    uint32_t a, b;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
    unpack8<T>(make_uint4(a, b, 0u, 0u), t);
  } else {
    uint32_t a;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(a) : "r"(addr));
    unpack8<T>(make_uint4(a, 0u, 0u, 0u), t);
  }
#pragma unroll
  for (int i = 0; i < DL; ++i) f[i] = t[i];
}

// --------------------------------------------------------------------------
// Merge of partial states (the reduce of src/kernel_triton.py:120-174).  A
// slot holds acc [G][D], m [G] (running max, log2 units) and l [G] (sum of
// 2^(score - m)); states combine by rescaling to the larger max.
// One warp folds R query-head rows at once: row r is spans [a[r], b[r])
// (a < b) of slots base[r] + j * sf, query head g[r].  Batches of SB spans
// per row are loaded together (each lane its NC float4 head-dim chunks
// c = 4 lane + 128 i, plus the span's m and l), then folded in span order
// with an online rescale into (M, L, acc).
template <int D, int R, int SB>
__device__ __forceinline__ void fold_rows(const float* const (&base)[R], const int (&g)[R],
                                          const int (&a)[R], const int (&b)[R], int sf, int G,
                                          int lane, float (&M)[R], float (&L)[R],
                                          float4 (&acc)[R][(D + 127) / 128]) {
  constexpr int NC = (D + 127) / 128;
  const int GD = G * D;
  int n = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    M[r] = -INFINITY;
    L[r] = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[r][c] = make_float4(0.f, 0.f, 0.f, 0.f);
    n = max(n, b[r] - a[r]);
  }
  for (int t0 = 0; t0 < n; t0 += SB) {
    float4 v[R][SB][NC];
    float mj[R][SB], lj[R][SB];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int u = 0; u < SB; ++u) {
        const int j = a[r] + t0 + u < b[r] ? a[r] + t0 + u : b[r] - 1;
        const float* ps = base[r] + static_cast<int64_t>(j) * sf;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const int cc = lane * 4 + 128 * c;
          v[r][u][c] = cc < D ? __ldcg(reinterpret_cast<const float4*>(ps + g[r] * D + cc))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        mj[r][u] = __ldcg(ps + GD + g[r]);
        lj[r][u] = __ldcg(ps + GD + G + g[r]);
      }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int u = 0; u < SB; ++u) {
        if (a[r] + t0 + u < b[r]) {
          const float mn = fmaxf(M[r], mj[r][u]);
          const float sa = fast_exp2(M[r] - mn), sb = fast_exp2(mj[r][u] - mn);
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            acc[r][c].x = acc[r][c].x * sa + v[r][u][c].x * sb;
            acc[r][c].y = acc[r][c].y * sa + v[r][u][c].y * sb;
            acc[r][c].z = acc[r][c].z * sa + v[r][u][c].z * sb;
            acc[r][c].w = acc[r][c].w * sa + v[r][u][c].w * sb;
          }
          L[r] = L[r] * sa + lj[r][u] * sb;
          M[r] = mn;
        }
      }
  }
}

// Writes a merged row: out (type T) or, in state mode, the fp32 state o and
// its lse (natural log).  acc holds the lane's chunks c = 4 lane + 128 i.
template <typename T, int D>
__device__ __forceinline__ void write_row(const DecodeParams& p, int hd, int g, int lane, float M,
                                          float L, const float4 (&acc)[(D + 127) / 128]) {
  const int G = p.G;
  const int s = hd / p.Hkv, h = hd - s * p.Hkv;
  const int Hq = p.Hkv * G, qh = h * G + g;
  const float inv = 1.f / L;
#pragma unroll
  for (int i = 0; i < (D + 127) / 128; ++i) {
    const int c = lane * 4 + 128 * i;
    if (c >= D) continue;
    const float4 a = acc[i];
    if (p.state_o) {
      *reinterpret_cast<float4*>(p.state_o + (static_cast<int64_t>(s) * Hq + qh) * D + c) =
          make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
    } else {
      T* o = static_cast<T*>(p.out) + s * p.o_sb + qh * p.o_sh + c;
      *reinterpret_cast<uint2*>(o) =
          make_uint2(pack2<T>(a.x * inv, a.y * inv), pack2<T>(a.z * inv, a.w * inv));
    }
  }
  if (p.state_o && lane == 0)
    p.state_lse[static_cast<int64_t>(s) * Hq + qh] = (M + __log2f(L)) * kLn2;
}

// --------------------------------------------------------------------------
// Decode kernel.  T: element type; D: head size; NT: query-head tiles of 8
// (G <= 8*NT); ST: tokens per ring stage (16, 32 or 64; a power of two
// >= block_size).  CORE selects CUDA-core arithmetic instead of tensor-core
// MMA for small query groups (G <= kCoreMaxG, ST == 32): one token per lane
// for q.K, a warp-shuffle softmax, lanes over the head dimension for P.V.
// PAIR splits a large query group over two warps that share one ring: the
// even warp of a pair (the leader) schedules, claims and issues every stage
// and computes query heads [0, 8 NT); the odd warp follows the stage records
// the leader writes, computes heads [8 NT, 16 NT), and releases each slot
// through a second mbarrier before the leader refills it (a sentinel record
// ends its loop).  Half the accumulator per warp halves the registers, so a
// group of up to 32 query heads fits at D = 128.  (At D = 64 the pair runs
// twice the resident warps of the single-warp kernel but is slower: each
// stage waits on both warps, and the per-stage issue work does not split.)
template <typename T, int D, int NT, int ST, bool CORE, bool PAIR = false, bool TC = false>
__global__ void __launch_bounds__(kMaxWarpsPerCta * 32, (PAIR && D == 64 && !TC) ? 2 : 1)
    decode_kernel(const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap,
                  const DecodeParams p) {
  constexpr int NH = D / 64;            // 128-byte planes per token row
  constexpr int LOG2_NH = NH == 1 ? 0 : (NH == 2 ? 1 : 2);
  constexpr int MT = ST / 16;           // 16-token MMA tiles per stage
  constexpr int LOG2_ST = ST == 16 ? 4 : (ST == 32 ? 5 : 6);
  constexpr int KS = D / 16;            // k-steps of QK^T == d-tiles of PV
  constexpr int PLANE = ST * 128;       // bytes of one plane of one stage
  constexpr int KV_BYTES = NH * PLANE;  // K (or V) bytes per stage
  constexpr int STAGE_BYTES = 2 * KV_BYTES;
  static_assert(D % 64 == 0 && (ST == 16 || ST == 32 || ST == 64), "shape");
  static_assert(!CORE || (ST == 32 && NT == 1 && D <= 128), "CUDA-core path shape");
  constexpr int DL = D / 32;  // head-dim elements per lane (CUDA-core path)
  static_assert(NH == 1 || NH == 2 || NH == 4, "head size");
  static_assert(!(CORE && PAIR), "the CUDA-core path has no paired variant");
  static_assert(!TC || (PAIR && !CORE && D == 64 && ST == 64 && NT == 2), "tcgen05 path shape");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t smem_base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (smem_base - raw_addr);

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int wpc = blockDim.x >> 5;
  const int depth = p.depth;
  // A "unit" owns one ring and one page range: a warp, or a pair of warps
  // (wpc is even for PAIR).  role 1 is the follower of a pair.
  const int role = PAIR ? (warp & 1) : 0;
  const int unit = PAIR ? (warp >> 1) : warp;
  const int upc = PAIR ? (wpc >> 1) : wpc;
  const int gw = blockIdx.x * upc + unit;
  const int g_lo = PAIR ? role * NT * 8 : 0;  // first query head of this warp
  const int n_heads = p.B * p.Hkv;
  // tcgen05 path: the query and probability tiles (shared by the two units
  // of a unit pair) follow the rings; the tail (mbarriers, stage records)
  // follows them.  Tensor memory is allocated once per CTA here, before any
  // early exit, and freed at the end of the kernel by the same warp after a
  // CTA barrier that every warp reaches.
  const int tc_tiles = TC ? ((upc + 1) / 2) * 2 * kTcTileBytes : 0;
  uint8_t* const tail0 = smem + upc * depth * STAGE_BYTES + tc_tiles;
  uint32_t tbase = 0;
  const uint32_t tc_cols = upc > 2 ? 512u : static_cast<uint32_t>(upc) * kTcUnitCols;
  if constexpr (TC) {
    const uint32_t slot = smem_addr(tail0) + tc_slot_offset(upc);
    if (warp == 0) {
      tmem_alloc(slot, tc_cols);
      tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tbase = *reinterpret_cast<volatile uint32_t*>(tail0 + tc_slot_offset(upc));
  }
  // The reduce grid may be scheduled at once: it waits for this grid to
  // complete before it reads anything.
  grid_launch_dependents();
  // Heads of length 0 get zeros (an empty state in state mode), matching
  // softmax over zero keys times an empty V in src/kernel_eager.py:51-53.
  // The planner lists them; this runs after the wait for the planner.
  auto zero_empty_heads = [&]() {
    const int n_empty = *p.n_empty;
    for (int e = gw; e < n_empty; e += p.total_warps) {
      const int hd = p.empty[e];
      const int s = hd / p.Hkv, h = hd - s * p.Hkv;
      const int Hq = p.Hkv * p.G;
      const int g_hi = PAIR ? min(p.G, g_lo + NT * 8) : p.G;
      for (int g = g_lo; g < g_hi; ++g) {
        const int qh = h * p.G + g;
        for (int c = lane * 4; c < D; c += 128) {
          if (p.state_o)
            *reinterpret_cast<float4*>(p.state_o + (static_cast<int64_t>(s) * Hq + qh) * D + c) =
                make_float4(0.f, 0.f, 0.f, 0.f);
          else
            *reinterpret_cast<uint2*>(static_cast<T*>(p.out) + s * p.o_sb + qh * p.o_sh + c) =
                make_uint2(0u, 0u);
        }
        if (p.state_o && lane == 0) p.state_lse[static_cast<int64_t>(s) * Hq + qh] = -INFINITY;
      }
    }
  };
  // Early start: the page-count prefix of every head, computed by this CTA
  // from the lengths (inputs: nothing the kernels before this one in the
  // stream write, as the host enables it only for calls without an append)
  // into shared memory — cum_sm [n_heads + 1], len_sm [n_heads] (clamped).
  // The planner computes the same prefix for the reduce kernel; both clamp
  // alike, so ranges, tail chunks and segments agree.  The tcgen05 path
  // keeps the prefix in its query / probability tiles, which it writes only
  // after every warp of the CTA has switched to the planner's copy (early
  // is cleared then).
  bool early = (!PAIR || TC) && p.early != 0;
  int* const cum_sm = reinterpret_cast<int*>(
      TC ? smem + upc * depth * STAGE_BYTES
         : tail0 + upc * kMaxDepth * (8 + kMetaBytesPerSlot) + upc * core_q_bytes(CORE, D));
  int* const len_sm = cum_sm + kEarlyMaxHeads + 1;
  int W, total, first_head = 0, sm_m, sm_k;
  if (early) {
    int* const wsum = len_sm + kEarlyMaxHeads;  // [32] per-warp sums
    const int nt = blockDim.x;
    const int per = (n_heads + nt - 1) / nt;
    const int h0 = threadIdx.x * per, h1 = min(h0 + per, n_heads);
    const int capl = p.maxb * p.bs;
    int sum = 0;
    for (int hd = h0; hd < h1; ++hd) {
      const int s = hd / p.Hkv, h = hd - s * p.Hkv;
      int L = p.lens[s * p.l_sb + h * p.l_sh];
      L = L < 0 ? 0 : (L > capl ? capl : L);
      len_sm[hd] = L;
      sum += (L + p.bs - 1) / p.bs;
    }
    int x = sum;  // inclusive scan within the warp, then across warps
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    int run = x - sum;
    for (int w = 0; w < warp; ++w) run += wsum[w];
    for (int hd = h0; hd < h1; ++hd) {
      cum_sm[hd] = run;
      run += (len_sm[hd] + p.bs - 1) / p.bs;
    }
    if (threadIdx.x == nt - 1) cum_sm[n_heads] = run;
    __syncthreads();
    total = cum_sm[n_heads];
    W = total < p.total_warps ? total : p.total_warps;
    tail_chunks(total, W, p.steal_m_max, p.steal_pps, p.steal_min_stages, &sm_m, &sm_k);
  } else {
    // Everything below reads what the planner wrote.  The start-up values
    // are independent loads, issued together (wstart has total_warps
    // entries, so the read is in bounds even for a warp that then exits).
    grid_dependency_wait();
    W = *p.weff;  // min(total_warps, total pages), set by the planner
    // Total pages < 2^31 (checked on the host), so page indices are 32-bit.
    total = p.cum[n_heads];
    first_head = gw < p.total_warps ? p.wstart[gw] : 0;
    const int4 steal = *reinterpret_cast<const int4*>(p.steal);
    sm_m = steal.x;
    sm_k = steal.y;
    zero_empty_heads();
  }
  const int gs = gw < W ? static_cast<int>(static_cast<int64_t>(gw) * total / W) : 0;
  const int g_end = gw < W ? static_cast<int>(static_cast<int64_t>(gw + 1) * total / W) : 0;
  // A unit without pages leaves (the tcgen05 path keeps it to the end, where
  // the CTA frees its tensor memory).
  const bool idle = gw >= W || total == 0 || gs >= g_end;
  if (idle) {
    if constexpr (!TC) {
      if (early) {
        grid_dependency_wait();
        zero_empty_heads();
      }
      return;
    }
  }
  // Current segment [c_gp, ge): the static prefix first, then tail chunks
  // claimed from the front of this warp's tail, then chunks stolen from the
  // back of other warps' tails.  run_start is the segment's first page.
  int ge = g_end - sm_m * sm_k;
  int run_start = gs;
  int mode = 0;  // 0: own range, 1: stealing, 2: no work left
  unsigned long long pend = 0ull;  // lane 0: result of the owner's claim
  bool claim_sent = false;

  const int G = p.G, Hkv = p.Hkv, bs = p.bs;
  const int log2_bs = __ffs(bs) - 1;          // bs is a power of two
  const int log2_pps = LOG2_ST - log2_bs;     // pages per stage = ST / bs
  const int pps = 1 << log2_pps;
  const int cap = p.maxb << log2_bs;
  const uint32_t ring = smem_base + unit * depth * STAGE_BYTES;
  uint8_t* tail = tail0;
  const uint32_t bars = smem_addr(tail) + unit * kMaxDepth * 8;
  int4* meta = reinterpret_cast<int4*>(tail + upc * kMaxDepth * 8) +
               unit * kMaxDepth * 2;
  float* qsm = reinterpret_cast<float*>(tail + upc * kMaxDepth * (8 + kMetaBytesPerSlot)) +
               unit * (core_q_bytes(CORE, D) / 4);
  // PAIR: "slot free" barriers, one arrival (the follower's) per phase.
  const uint32_t empties = smem_addr(tail) + upc * kMaxDepth * (8 + kMetaBytesPerSlot) +
                           upc * core_q_bytes(CORE, D) + unit * kMaxDepth * 8;

  // tcgen05 path, per unit: scores of even / odd stages ready (MMA
  // commit), probabilities-times-V of a stage done (MMA commit; frees the
  // probability tile, the stage's ring slot and the output accumulator),
  // probabilities written (one arrival per warp), and one drain barrier per
  // warp (MMA commit).
  const uint32_t tcb = smem_addr(tail) + tc_bars_offset(upc) + unit * kTcBarsPerUnit * 8;
  if (lane == 0 && role == 0) {
    for (int i = 0; i < depth; ++i) {
      mbar_init(bars + i * 8, 1);
      if constexpr (PAIR) mbar_init(empties + i * 8, 1);
    }
    if constexpr (TC) {
      mbar_init(tcb, 1);
      mbar_init(tcb + 8, 1);
      mbar_init(tcb + 16, 1);
      mbar_init(tcb + 24, 2);
      mbar_init(tcb + 32, 1);
      mbar_init(tcb + 40, 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if constexpr (PAIR) {
    // The pair's barriers are initialised.  Fixed barrier ids (one per
    // ring; upc <= kMaxWarpsPerCta / 2 = 4) keep the count ptxas reserves low.
    static_assert(kMaxWarpsPerCta / 2 <= 4, "one named barrier per ring");
    switch (unit) {
      case 0: named_barrier_sync<1>(64); break;
      case 1: named_barrier_sync<2>(64); break;
      case 2: named_barrier_sync<3>(64); break;
      default: named_barrier_sync<4>(64); break;
    }
  } else {
    __syncwarp();
  }
  const uint64_t policy = l2_policy_evict_first();

  // ------------------------------------------------ issue-side cursor state
  // Window of 32 consecutive heads starting at `win`: lane i holds cum[win+i]
  // and the clamped length of head win+i.
  int win = 0;
  int win_cum = 0, win_len = 0;
  auto load_window = [&](int w0) {
    win = w0;
    const int hd = w0 + lane;
    if (early) {
      win_cum = (hd <= n_heads) ? cum_sm[hd] : 0;
      win_len = (hd < n_heads) ? len_sm[hd] : 0;
      return;
    }
    win_cum = (hd <= n_heads) ? p.cum[hd] : 0;
    int L = 0;
    if (hd < n_heads) {
      const int s = hd / Hkv, h = hd - s * Hkv;
      L = p.lens[s * p.l_sb + h * p.l_sh];
      L = L < 0 ? 0 : (L > cap ? cap : L);
    }
    win_len = L;
  };
  int c_gp = gs;  // next global page to stage
  // Current head of the issue cursor and what the stages of it need.
  int c_head = 0, c_h = 0, c_lo = 0, c_hi = 0, c_len = 0, c_slot = 0, c_vfirst = 0, c_vlast = 0;
  const int32_t* c_bt = p.bt;
  int64_t c_pid_add = 0;
  auto enter_head = [&](int hd) {
    if (hd + 1 - win > 31) load_window(hd);
    c_head = hd;
    c_lo = __shfl_sync(0xffffffffu, win_cum, hd - win);
    c_hi = __shfl_sync(0xffffffffu, win_cum, hd + 1 - win);
    c_len = __shfl_sync(0xffffffffu, win_len, hd - win);
    if (c_hi > c_lo) {
      const int s = hd / Hkv;
      c_h = hd - s * Hkv;
      c_bt = p.bt + s * p.bt_sb + c_h * p.bt_sh;
      c_pid_add = static_cast<int64_t>(c_h) * p.bt_add;
      c_vfirst = segment_of_page(c_lo, total, W, sm_m, sm_k);
      c_vlast = segment_of_page(c_hi - 1, total, W, sm_m, sm_k);
      c_slot = segment_of_page(c_lo > run_start ? c_lo : run_start, total, W, sm_m, sm_k);
    }
  };
  // Largest head hd with cum[hd] <= P (the head holding global page P):
  // 32 probes per round narrow the range 32-fold.
  auto find_head = [&](int P) -> int {
    int lo = 0, hi = n_heads;
    while (hi - lo > 1) {
      const int step = (hi - lo + 31) / 32;
      const int x = lo + lane * step;
      // true for lane 0: cum[lo] <= P
      const bool le = x < hi && (early ? cum_sm[x] : p.cum[x]) <= P;
      const unsigned mask = __ballot_sync(0xffffffffu, le);
      lo += (31 - __clz(mask)) * step;
      hi = lo + step < hi ? lo + step : hi;
    }
    return lo;
  };
  if (early) first_head = find_head(gs);
  load_window(first_head);
  enter_head(win);
  // Claim a tail chunk of another warp (from the back of its tail).  Each
  // round reads the claim words of 32 warps picked by a shared cursor and
  // tries the one with the most chunks left; gives up once the planner's
  // count of unclaimed chunks reaches zero or after a bounded number of
  // rounds.  Returns the chunk's first page, or -1.
  auto steal_chunk = [&]() -> int {
    const int rounds = 2 * ((W + 31) / 32) + 2;
    for (int r = 0; r < rounds; ++r) {
      int left = 0;
      uint32_t c0 = 0;
      if (lane == 0) {
        left = *reinterpret_cast<volatile int32_t*>(p.steal + 2);
        c0 = atomicAdd(reinterpret_cast<unsigned int*>(p.steal + 3), 32u);
      }
      left = __shfl_sync(0xffffffffu, left, 0);
      if (left <= 0) return -1;
      c0 = __shfl_sync(0xffffffffu, c0, 0);
      const int v = static_cast<int>((c0 + lane) % static_cast<uint32_t>(W));
      const unsigned long long wd =
          *reinterpret_cast<volatile unsigned long long*>(p.claims + v);
      const int used = static_cast<int>(static_cast<uint32_t>(wd)) +
                       static_cast<int>(static_cast<uint32_t>(wd >> 32));
      const int rem = used < sm_m ? sm_m - used : 0;
      int key = (rem << 5) | (31 - lane);  // most left, then lowest lane
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
      if ((key >> 5) == 0) continue;
      const int vb = __shfl_sync(0xffffffffu, v, 31 - (key & 31));
      unsigned long long old = 0ull;
      if (lane == 0) old = atomicAdd(p.claims + vb, 1ull << 32);
      old = __shfl_sync(0xffffffffu, old, 0);
      const uint32_t f = static_cast<uint32_t>(old), b = static_cast<uint32_t>(old >> 32);
      if (f + b < static_cast<uint32_t>(sm_m)) {
        if (lane == 0) atomicSub(p.steal + 2, 1);
        const int a1 = static_cast<int>(static_cast<int64_t>(vb + 1) * total / W);
        return a1 - static_cast<int>(b + 1) * sm_k;  // chunk m - b (1-based)
      }
    }
    return -1;
  };
  // The current segment is used up: move to this warp's next tail chunk
  // (which starts where the segment ended) or to a stolen one.  The owner's
  // claim is sent with the segment's last stage, not earlier, so that a slow
  // warp keeps no chunk reserved that a faster one could take.
  auto next_region = [&]() -> bool {
    if (mode == 0) {
      if (sm_m > 0) {
        if (!claim_sent && lane == 0) pend = atomicAdd(p.claims + gw, 1ull);
        claim_sent = false;
        const unsigned long long old = __shfl_sync(0xffffffffu, pend, 0);
        const uint32_t f = static_cast<uint32_t>(old), b = static_cast<uint32_t>(old >> 32);
        if (f + b < static_cast<uint32_t>(sm_m)) {
          run_start = ge;  // chunk f + 1
          ge += sm_k;
          if (c_gp < c_hi)
            c_slot = segment_of_page(run_start, total, W, sm_m, sm_k);
          if (lane == 0) atomicSub(p.steal + 2, 1);
          return true;
        }
      }
      mode = 1;
    }
    if (mode == 1) {
      const int cs = sm_m > 0 ? steal_chunk() : -1;
      if (cs >= 0) {
        c_gp = cs;
        ge = cs + sm_k;
        run_start = cs;
        const int hd = find_head(cs);
        load_window(hd);
        enter_head(hd);
        return true;
      }
      mode = 2;
    }
    return false;
  };

  // Early start: the warp streams and computes without waiting for the
  // planner (and, through it, for the previous call's reduce kernel) until
  // its first action on shared state — an output or partial-state write, a
  // tail-chunk claim, a status bit — and waits for it only then.  Until
  // then a bad page id is remembered, not yet reported: the planner resets
  // the status word.
  bool prewait = early;
  bool pending_bad = false;
  auto ensure_waited = [&]() {
    if (!prewait) return;
    grid_dependency_wait();
    prewait = false;
    if (pending_bad && lane == 0) atomicOr(p.status, kStatusBadPage);
    zero_empty_heads();
  };
  // Next stage, prepared one issue ahead so its block-table loads overlap.
  bool nx_valid = false;
  int nx_head = 0, nx_h = 0, nx_lp0 = 0, nx_np = 0, nx_len = 0, nx_slot = 0, nx_vfirst = 0,
      nx_vlast = 0;
  // lane i < nx_np: block-table entry of page i of the stage, kept as
  // loaded (the page id is formed where it is used, one stage later, so the
  // load's latency is not waited for here), and the head's page-id offset.
  int32_t nx_raw = 0;
  int64_t nx_add = 0;
  auto prepare_next = [&]() {
    if (c_gp >= ge) {
      ensure_waited();  // claims and stealing touch shared state
      if (!next_region()) {
        nx_valid = false;
        return;
      }
    }
    while (c_gp >= c_hi) enter_head(c_head + 1);
    nx_valid = true;
    nx_head = c_head;
    nx_h = c_h;
    nx_lp0 = c_gp - c_lo;
    int np = pps;
    if (c_hi - c_gp < np) np = c_hi - c_gp;
    if (ge - c_gp < np) np = ge - c_gp;
    nx_np = np;
    // The segment's last stage: claim this warp's next tail chunk now, so the
    // atomic completes while the stages in flight are computed.
    if (mode == 0 && sm_m > 0 && !claim_sent && c_gp + np >= ge) {
      ensure_waited();
      if (lane == 0) pend = atomicAdd(p.claims + gw, 1ull);
      claim_sent = true;
    }
    nx_len = c_len;
    nx_slot = c_slot;
    nx_vfirst = c_vfirst;
    nx_vlast = c_vlast;
    if (lane < np)
      nx_raw = c_bt[static_cast<int64_t>(nx_lp0 + lane) * p.bt_si];
    nx_add = c_pid_add;
    c_gp += np;
  };
  auto issue = [&](int slot) -> bool {
    if (!nx_valid) return false;
    const uint32_t bar = bars + slot * 8;
    if (lane == 0) {
      meta[slot * 2] = make_int4(nx_head, nx_lp0, nx_np, nx_len);
      meta[slot * 2 + 1] = make_int4(nx_slot, 0, nx_vfirst, nx_vlast);
      mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nx_np << (log2_bs + LOG2_NH + 8)));
    }
    __syncwarp();
    const int64_t nx_pid = static_cast<int64_t>(nx_raw) * p.bt_mul + nx_add;
    const bool bad = lane < nx_np && (nx_pid < 0 || nx_pid >= p.num_pages);
    if (__any_sync(0xffffffffu, bad)) {
      if (prewait)
        pending_bad = true;
      else if (lane == 0)
        atomicOr(p.status, kStatusBadPage);
    }
    // A rejected page id reads a box that lies wholly outside the tensor
    // (negative row), which the TMA unit fills with zeros.
    const int32_t row = bad ? -256 : (static_cast<int32_t>(nx_pid) << log2_bs);
    // lane -> (K or V, page of the stage, 64-column plane)
    const int kv = lane >> (log2_pps + LOG2_NH);
    const int pg = (lane >> LOG2_NH) & (pps - 1);
    const int hf = lane & (NH - 1);
    const int32_t zrow = __shfl_sync(0xffffffffu, row, pg);
    if (kv < 2 && pg < nx_np) {
      const uint32_t dst = ring + slot * STAGE_BYTES + kv * KV_BYTES + hf * PLANE +
                           (pg << (log2_bs + 7));
      tma_load_3d(dst, kv ? &vmap : &kmap, hf * 64, p.head_in_map ? nx_h : 0, zrow, bar,
                  policy);
    }
    prepare_next();
    return true;
  };

  // ------------------------------------------------ compute-side state
  const int lr = lane >> 2;  // fragment row group
  const int lc = lane & 3;   // fragment column pair
  const int x7 = lane & 7;
  const uint32_t k_lane = static_cast<uint32_t>(((lane & 7) + ((lane >> 3) & 1) * 8) * 128);
  const int k_chunk = lane >> 4;
  const uint32_t v_lane = static_cast<uint32_t>(((lane & 7) + (lane >> 4) * 8) * 128);
  const int v_chunk = (lane >> 3) & 1;
  const float scale_log2 = p.scale_log2;

  uint32_t qb[KS][NT][2];
  float acc[KS][NT][4];
  float mrun[NT][2], lrun[NT][2];
  // CUDA-core path: lane owns head-dim elements [lane*DL, lane*DL + DL) of
  // every query head; cm is the running max (log2 units, warp-uniform), cl
  // this lane's part of the running sum.
  float cacc[kCoreMaxG][DL];
  float cm[kCoreMaxG], cl[kCoreMaxG];

  // Resets the running state for a new segment of head `hd`; loads the
  // head's query group unless it is already in place (same head).
  auto start_head = [&](int hd, bool load_q) {
    const int s = hd / Hkv, h = hd - s * Hkv;
    const T* qp = static_cast<const T*>(p.q) + s * p.q_sb + static_cast<int64_t>(h) * G * p.q_sh;
    if constexpr (CORE) {
      if (load_q) {
        __syncwarp();  // the previous head's q is no longer read
        for (int idx = lane; idx < kCoreMaxG * D; idx += 32) {
          const int g = idx / D, d = idx - g * D;
          qsm[idx] = g < G ? static_cast<float>(qp[g * p.q_sh + d]) : 0.f;
        }
        __syncwarp();
      }
#pragma unroll
      for (int g = 0; g < kCoreMaxG; ++g) {
        cm[g] = -INFINITY;
        cl[g] = 0.f;
#pragma unroll
        for (int e = 0; e < DL; ++e) cacc[g][e] = 0.f;
      }
    } else {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int g = g_lo + nt * 8 + lr;
      if (load_q) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t b0 = 0, b1 = 0;
          if (g < G) {
            const T* row = qp + g * p.q_sh + ks * 16 + lc * 2;
            b0 = *reinterpret_cast<const uint32_t*>(row);
            b1 = *reinterpret_cast<const uint32_t*>(row + 8);
          }
          qb[ks][nt][0] = b0;
          qb[ks][nt][1] = b1;
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        mrun[nt][e] = -INFINITY;
        lrun[nt][e] = 0.f;
      }
#pragma unroll
      for (int dt = 0; dt < KS; ++dt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[dt][nt][i] = 0.f;
    }
    }  // CORE / MMA state
  };

  // Ends the accumulation of head `hd` in segment `slot`: a head wholly
  // inside one segment (vfirst == vlast) is written directly; otherwise the
  // segment's part becomes the partial state in slot hd + `slot` (plain
  // stores: a reduce kernel merges the head's slots after this grid).
  auto finish_head = [&](int hd, int slot, int vfirst, int vlast) {
    ensure_waited();  // outputs and partial slots of the previous call
    const bool whole = vfirst == vlast;
    if constexpr (CORE) {
      const int s = hd / Hkv, h = hd - s * Hkv;
      const int Hq = Hkv * G;
      float lt[kCoreMaxG];
#pragma unroll
      for (int g = 0; g < kCoreMaxG; ++g) {
        float l = cl[g];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        lt[g] = l;
      }
      const int d0 = lane * DL;
      if (whole) {
#pragma unroll
        for (int g = 0; g < kCoreMaxG; ++g) {
          if (g >= G) break;
          const float inv = 1.f / lt[g];
          const int qh = h * G + g;
          if (p.state_o) {
            float* o = p.state_o + (static_cast<int64_t>(s) * Hq + qh) * D + d0;
#pragma unroll
            for (int e = 0; e < DL; ++e) o[e] = cacc[g][e] * inv;
            if (lane == 0)
              p.state_lse[static_cast<int64_t>(s) * Hq + qh] = (cm[g] + __log2f(lt[g])) * kLn2;
          } else {
            T* o = static_cast<T*>(p.out) + s * p.o_sb + qh * p.o_sh + d0;
#pragma unroll
            for (int e = 0; e < DL; e += 2)
              *reinterpret_cast<uint32_t*>(o + e) = pack2<T>(cacc[g][e] * inv, cacc[g][e + 1] * inv);
          }
        }
        return;
      }
      float* ps = p.part + static_cast<int64_t>(hd + slot) * p.slot_floats;
#pragma unroll
      for (int g = 0; g < kCoreMaxG; ++g) {
        if (g >= G) break;
#pragma unroll
        for (int e = 0; e < DL; ++e) __stcg(ps + g * D + d0 + e, cacc[g][e]);
        if (lane == 0) {
          __stcg(ps + G * D + g, cm[g]);
          __stcg(ps + G * D + G + g, lt[g]);
        }
      }
    } else {
    float lt[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float l = lrun[nt][e];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        lt[nt][e] = l;
      }
    const int s = hd / Hkv, h = hd - s * Hkv;
    const int Hq = Hkv * G;
    if (whole) {
      float inv[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) inv[nt][e] = 1.f / lt[nt][e];
#pragma unroll
      for (int dt = 0; dt < KS; ++dt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int g = g_lo + nt * 8 + lc * 2 + (i & 1);
            const int d = dt * 16 + lr + (i >> 1) * 8;
            if (g < G) {
              const float v = acc[dt][nt][i] * inv[nt][i & 1];
              const int qh = h * G + g;
              if (p.state_o)
                p.state_o[(static_cast<int64_t>(s) * Hq + qh) * D + d] = v;
              else
                static_cast<T*>(p.out)[s * p.o_sb + qh * p.o_sh + d] = from_float<T>(v);
            }
          }
      if (p.state_o && lr == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int g = g_lo + nt * 8 + lc * 2 + e;
            if (g < G)
              p.state_lse[static_cast<int64_t>(s) * Hq + h * G + g] =
                  (mrun[nt][e] + __log2f(lt[nt][e])) * kLn2;
          }
      }
      return;
    }
    // Split head: publish this segment's partial.
    float* ps = p.part + static_cast<int64_t>(hd + slot) * p.slot_floats;
#pragma unroll
    for (int dt = 0; dt < KS; ++dt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int g = g_lo + nt * 8 + lc * 2 + (i & 1);
          const int d = dt * 16 + lr + (i >> 1) * 8;
          if (g < G) __stcg(ps + g * D + d, acc[dt][nt][i]);
        }
    if (lr == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int g = g_lo + nt * 8 + lc * 2 + e;
          if (g < G) {
            __stcg(ps + G * D + g, mrun[nt][e]);
            __stcg(ps + G * D + G + g, lt[nt][e]);
          }
        }
    }
    }  // CORE / MMA partial publication
  };

  // ------------------------------------------------ pipeline
  int issued = 0;          // stages issued (leader)
  bool sent_end = false;   // PAIR leader: the follower's end record is out
  // PAIR: the record of stage `issued` in (free) slot `slot` says "no more
  // stages"; a plain arrival completes the slot's phase.
  auto send_end = [&](int slot) {
    if (lane == 0) {
      meta[slot * 2] = make_int4(-1, 0, 0, 0);
      mbar_arrive(bars + slot * 8);
    }
    sent_end = true;
  };
  if constexpr (TC) {
    // ------------------------------------------- tcgen05 pipeline (a unit)
    // Stage it: S = Q K^T on the tensor core as two 64 x 32 halves (tokens
    // 0-31 and 32-63 of the stage), written to the lower and the upper 16
    // lanes of every TMEM sub-partition, so that each thread of a warp owns
    // one (query head, 32-token half) of the scores.  The warps turn them
    // into probabilities (online softmax in fp32, log2 units) stored to the
    // probability tile, and O += P V accumulates in TMEM (64 columns).  Lane
    // 0 of the MMA warp issues every MMA; the scores of stage it + 1 are
    // computed while the warps work on stage it.
    //
    // The MMAs have M = 64 rows: rows 0-31 belong to even units, rows 32-63
    // to odd units (a warp reads only its own TMEM sub-partition, warp % 4;
    // row r of an M = 64 accumulator lies in lane (r % 16) + 32 (r / 16), 16
    // lanes higher for the upper half).  The query and probability tiles of
    // a unit pair are shared, each unit writing its own 32 rows; the rows of
    // the other unit only produce accumulator rows that nobody reads.
    constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    // Instruction descriptors: fp32 accumulate, A and B of type T, M = 64;
    // QK^T with both operands K-major and N = 32; PV with B (V) MN-major and
    // N = 64.
    constexpr uint32_t kIdescQK =
        (1u << 4) | (kFmt << 7) | (kFmt << 10) | ((32u >> 3) << 17) | ((64u >> 4) << 24);
    constexpr uint32_t kIdescPV = (1u << 4) | (kFmt << 7) | (kFmt << 10) | (1u << 16) |
                                  ((64u >> 3) << 17) | ((64u >> 4) << 24);
    // mbarriers: scores ready (two buffers), PV done, probabilities written,
    // then one drain barrier per warp.
    const uint32_t sfull0 = tcb, ofree = tcb + 16, pready = tcb + 24, drain = tcb + 32;
    const uint32_t tiles = smem_base + upc * depth * STAGE_BYTES;
    const uint32_t qtile = tiles + (unit >> 1) * kTcTileBytes;
    const uint32_t ptile = tiles + ((upc + 1) / 2 + (unit >> 1)) * kTcTileBytes;
    const int quad = warp & 3;
    const uint32_t t_lane = static_cast<uint32_t>(32 * quad) << 16;
    const uint32_t ucol = tbase + unit * kTcUnitCols;
    const int row = 16 * quad + (lane & 15);  // this thread's row of the 64-row tiles
    const int g_row = row - 32 * (unit & 1);  // its query head
    const int half = lane >> 4;               // its 32 tokens of a stage
    // Waits whose outcome the whole warp shares (the tcgen05 loads, stores
    // and allocations below are warp-collective).
    auto wait_w = [&](uint32_t bar, uint32_t par) {
      return __all_sync(0xffffffffu, mbar_wait(bar, par, kWaitLimitNs));
    };
    // MMA warp: this unit's 32 query rows of the tile (zeros past G).  With
    // 16-byte aligned rows, lane l loads 16-byte chunk l % 8 of rows
    // 4 i + l / 8 (coalesced, all loads in flight at once); otherwise each
    // lane loads its row in 4-byte words.
    const bool q_vec = (reinterpret_cast<uintptr_t>(p.q) & 15) == 0 && (p.q_sb & 7) == 0 &&
                       (p.q_sh & 7) == 0;
    auto load_q = [&](int hd) {
      const int s = hd / Hkv, h = hd - s * Hkv;
      const T* qh0 = static_cast<const T*>(p.q) + s * p.q_sb + static_cast<int64_t>(h) * G * p.q_sh;
      const int rbase = 32 * (unit & 1);
      if (q_vec) {
        uint4 w[8];
        const int c = lane & 7;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int g = 4 * i + (lane >> 3);
          w[i] = g < G ? *reinterpret_cast<const uint4*>(qh0 + g * p.q_sh + c * 8)
                       : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = rbase + 4 * i + (lane >> 3);
          st_shared_v4(qtile + r * 128 + static_cast<uint32_t>((c ^ (r & 7)) << 4), w[i].x, w[i].y,
                       w[i].z, w[i].w);
        }
      } else {
        const int r = rbase + lane;
        uint32_t w[32];
        if (lane < G) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(qh0 + lane * p.q_sh);
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = src[i];
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = 0u;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(qtile + r * 128 + static_cast<uint32_t>((c ^ (r & 7)) << 4), w[4 * c],
                       w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
      }
      fence_proxy_async_smem();  // generic writes, read by the tensor core
      __syncwarp();
    };
    // Shared-memory descriptors (128-byte swizzle, 8-row groups 1024 bytes
    // apart) of the query tile, the probability tile and slot 0 of the
    // ring; an operand at byte offset o adds o >> 4 (no carry out of the
    // 14-bit start address: shared addresses are below 256 KB).
    const uint64_t qdesc = smem_desc_sw128(qtile, 16, 1024);
    const uint64_t pdesc = smem_desc_sw128(ptile, 16, 1024);
    const uint64_t rdesc = smem_desc_sw128(ring, 16, 1024);
    // MMA warp: S(j) = Q K(j)^T into score buffer j & 1 (K-steps of 16
    // elements advance 32 bytes inside the swizzled rows; tokens 32-63 of
    // the stage start 32 rows on).
    auto issue_qk = [&](int j) {
      const uint64_t kd = rdesc + static_cast<uint32_t>(((j % depth) * STAGE_BYTES) >> 4);
      const uint32_t d = ucol + (j & 1) * 32;
      if (lane == 0) {
        tc_fence_after();
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc_mma_ss(d + (static_cast<uint32_t>(hf) << 20), qdesc + ks * 2,
                      kd + (hf * 4096 + ks * 32) / 16, kIdescQK, static_cast<uint32_t>(ks));
        tc_commit(sfull0 + (j & 1) * 8);
      }
      __syncwarp();
    };
    // MMA warp: O (+)= P V(j) (K-steps of 16 tokens: 32 bytes along the
    // probability rows, 16 rows = 2048 bytes down V).
    auto issue_pv = [&](int j, bool accumulate) {
      const uint64_t vd = rdesc + static_cast<uint32_t>(((j % depth) * STAGE_BYTES + KV_BYTES) >> 4);
      if (lane == 0) {
        tc_fence_after();
#pragma unroll
        for (int kt = 0; kt < 4; ++kt)
          tc_mma_ss(ucol + 64, pdesc + kt * 2, vd + kt * 128, kIdescPV,
                    (accumulate || kt > 0) ? 1u : 0u);
        tc_commit(ofree);
      }
      __syncwarp();
    };
    float m_run = -INFINITY, l_run = 0.f;  // this row's running max and this thread's sum
    // Ends head hd's accumulation in segment `slot` (after its last PV):
    // lanes 0-15 hold the rows of the output accumulator.
    auto tc_finish = [&](int hd, int slot, int vfirst, int vlast) {
      ensure_waited();
      const float lt = l_run + __shfl_xor_sync(0xffffffffu, l_run, 16);
      uint32_t o[64];
      tmem_ld64(t_lane + ucol + 64, o);
      tmem_wait_ld();
      if (lane >= 16 || g_row >= G) return;
      const int s = hd / Hkv, h = hd - s * Hkv;
      const int Hq = Hkv * G, qh = h * G + g_row;
      if (vfirst == vlast) {
        const float inv = 1.f / lt;
        if (p.state_o) {
          float* dst = p.state_o + (static_cast<int64_t>(s) * Hq + qh) * D;
#pragma unroll
          for (int c = 0; c < 16; ++c)
            *reinterpret_cast<float4*>(dst + 4 * c) =
                make_float4(__uint_as_float(o[4 * c]) * inv, __uint_as_float(o[4 * c + 1]) * inv,
                            __uint_as_float(o[4 * c + 2]) * inv, __uint_as_float(o[4 * c + 3]) * inv);
          p.state_lse[static_cast<int64_t>(s) * Hq + qh] = (m_run + __log2f(lt)) * kLn2;
        } else {
          T* dst = static_cast<T*>(p.out) + s * p.o_sb + qh * p.o_sh;
#pragma unroll
          for (int c = 0; c < 16; ++c)
            *reinterpret_cast<uint2*>(dst + 4 * c) =
                make_uint2(pack2<T>(__uint_as_float(o[4 * c]) * inv, __uint_as_float(o[4 * c + 1]) * inv),
                           pack2<T>(__uint_as_float(o[4 * c + 2]) * inv, __uint_as_float(o[4 * c + 3]) * inv));
        }
        return;
      }
      float* ps = p.part + static_cast<int64_t>(hd + slot) * p.slot_floats;
#pragma unroll
      for (int c = 0; c < 16; ++c)
        __stcg(reinterpret_cast<float4*>(ps + g_row * D + 4 * c),
               make_float4(__uint_as_float(o[4 * c]), __uint_as_float(o[4 * c + 1]),
                           __uint_as_float(o[4 * c + 2]), __uint_as_float(o[4 * c + 3])));
      __stcg(ps + G * D + g_row, m_run);
      __stcg(ps + G * D + G + g_row, lt);
    };

    // Roles: warp 0 of the unit loads the queries and issues every MMA;
    // warp 1 produces the stages (schedule, tail-chunk claims, copies, stage
    // records) and refills the slot the previous PV freed after publishing
    // its probability rows, so that the refill overlaps the MMAs.  Both
    // compute the softmax of their 32 rows.
    const bool producer = role == 1;
    bool failed = false;
    int fw = 0;         // MMA warp: stages whose scores it has issued
    int waited = 0;     // producer: stages whose copies it has waited for
    int q_head = -1;    // MMA warp: the head whose queries are in the tile
    int n_done = 0;     // stages processed
    int cur_head = -1, cur_slot = -1, cur_vfirst = 0, cur_vlast = 0;
    // MMA warp: the scores of stage j (its copies have landed), unless its
    // record is the end record.
    auto start_qk = [&](int j) {
      fw = j + 1;
      const int hj = meta[(j % depth) * 2].x;
      if (hj < 0) return;
      if (hj != q_head) {
        q_head = hj;
        load_q(hj);
      }
      issue_qk(j);
    };
    // Prologue: the producers issue their first stages (on an early start,
    // from the prefix in shared memory, before the planner has finished);
    // then every warp waits for the plan and reads the prefix from global
    // memory from here on, and a CTA barrier orders those reads before any
    // tile write and publishes the first stage records, so that the MMA
    // warps load the first head's queries while the first copies are in
    // flight.  No warp waits on anything before the barrier except the
    // plan.
    if (!idle && producer) {
      prepare_next();
      for (int i = 0; i < depth; ++i) {
        if (!issue(i)) {
          send_end(i);
          break;
        }
        ++issued;
      }
    }
    ensure_waited();
    early = false;
    __syncthreads();
    if (!idle) {
      if (!producer) {
        const int h0 = meta[0].x;
        if (h0 >= 0) {
          q_head = h0;
          load_q(h0);
        }
        if (wait_w(bars, 0u))
          start_qk(0);
        else
          failed = true;
      }
      for (int it = 0; !failed; ++it) {
        if (producer && it >= issued) break;
        const int slot = it % depth;
        // The stage's copies have landed; its record (or the end record,
        // for the MMA warp) is visible.
        if (!wait_w(bars + slot * 8, static_cast<uint32_t>((it / depth) & 1))) {
          failed = true;
          break;
        }
        if (producer) waited = it + 1;
        const int4 m0 = meta[slot * 2];
        const int4 m1 = meta[slot * 2 + 1];
        if (m0.x < 0) break;  // end record (MMA warp)
        const bool new_seg = m0.x != cur_head || m1.x != cur_slot;
        bool o_done = it == 0;  // PV of the previous stage complete
        if (new_seg) {
          if (cur_head >= 0) {
            if (!wait_w(ofree, static_cast<uint32_t>((it - 1) & 1))) {
              failed = true;
              break;
            }
            tc_fence_after();
            o_done = true;
            tc_finish(cur_head, cur_slot, cur_vfirst, cur_vlast);
          }
          cur_head = m0.x;
          cur_slot = m1.x;
          cur_vfirst = m1.z;
          cur_vlast = m1.w;
          m_run = -INFINITY;
          l_run = 0.f;
        }
        if (!wait_w(sfull0 + (it & 1) * 8, static_cast<uint32_t>((it >> 1) & 1))) {
          failed = true;
          break;
        }
        tc_fence_after();
        uint32_t sr[32];
        tmem_ld32(t_lane + ucol + (it & 1) * 32, sr);
        tmem_wait_ld();
        // MMA warp: the next stage's scores now if its copies have landed
        // (else after this stage's PV), so that they are ready when this
        // stage is done.  The score buffer they overwrite was read by both
        // warps before their arrivals for stage it - 1, which this warp
        // waited for before that stage's PV.
        if (!producer && fw < it + 2 &&
            __all_sync(0xffffffffu, mbar_test_wait(bars + ((it + 1) % depth) * 8,
                                                   static_cast<uint32_t>(((it + 1) / depth) & 1))))
          start_qk(it + 1);
        // Scores in log2 units; tokens past the stage's valid count masked.
        const int ntok_stage = m0.z << log2_bs;
        const int ntok_left = m0.w - (m0.y << log2_bs);
        const int ntok = ntok_stage < ntok_left ? ntok_stage : ntok_left;
        float sv[32];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[i] = half * 32 + i < ntok ? __uint_as_float(sr[i]) * scale_log2 : -INFINITY;
          mx = fmaxf(mx, sv[i]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        // Lazy rescale: the running max moves only when a stage's max
        // exceeds it by more than 8 (log2 units), so probabilities stay
        // below 2^8 and the accumulator is rarely rescaled; the state (m,
        // acc, l) is exact for any m.
        const bool raise = mx > m_run + 8.f;  // always on a segment's first stage
        const bool rescale = raise && m_run != -INFINITY;
        const float m_new = raise ? mx : m_run;
        const float alpha = rescale ? fast_exp2(m_run - m_new) : 1.f;
        // Probabilities (type T), computed before the previous PV is waited for.
        float ls = 0.f;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = fast_exp2(sv[2 * i] - m_new);
          const float p1 = fast_exp2(sv[2 * i + 1] - m_new);
          ls += p0 + p1;
          pk[i] = pack2<T>(p0, p1);
        }
        l_run = l_run * alpha + ls;
        m_run = m_new;
        // The previous stage's PV is done: the probability tile and the
        // accumulator may be written, and its slot refilled.
        if (!o_done) {
          if (!wait_w(ofree, static_cast<uint32_t>((it - 1) & 1))) {
            failed = true;
            break;
          }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale)) {
          uint32_t o[64];
          tmem_ld64(t_lane + ucol + 64, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 64; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st64(t_lane + ucol + 64, o);
          tmem_wait_st();
        }
        // This unit's rows of the probability tile.
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = half * 4 + j;
          st_shared_v4(ptile + row * 128 + static_cast<uint32_t>((c ^ (row & 7)) << 4), pk[4 * j],
                       pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        }
        // V rows past the valid tokens may hold stale or non-finite data:
        // zero them so that 0 * V stays 0 (whole 128-byte rows).
        if (ntok < ST) {
          uint4* vz = reinterpret_cast<uint4*>(smem + (ring - smem_base) + slot * STAGE_BYTES + KV_BYTES);
          for (int idx = role * 32 + lane; idx < (ST - ntok) * 8; idx += 64)
            vz[(ntok + (idx >> 3)) * 8 + (idx & 7)] = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();  // P and V writes, read by the tensor core
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pready);
        n_done = it + 1;
        if (producer) {
          // The previous stage's slot is free (its PV is done).
          if (it > 0 && !sent_end) {
            const int fs = (it - 1) % depth;
            if (issue(fs))
              ++issued;
            else
              send_end(fs);
          }
        } else {
          // Both warps' probability rows are in place: O (+)= P V.
          if (!wait_w(pready, static_cast<uint32_t>(it & 1))) {
            failed = true;
            break;
          }
          issue_pv(it, !new_seg);
          if (fw < it + 2) {
            if (!wait_w(bars + ((it + 1) % depth) * 8, static_cast<uint32_t>(((it + 1) / depth) & 1))) {
              failed = true;
              break;
            }
            start_qk(it + 1);
          }
        }
      }
      // The last segment, after its last PV.
      if (!failed && cur_head >= 0) {
        if (wait_w(ofree, static_cast<uint32_t>((n_done - 1) & 1))) {
          tc_fence_after();
          tc_finish(cur_head, cur_slot, cur_vfirst, cur_vlast);
        } else {
          failed = true;
        }
      }
      if (failed) {
        ensure_waited();
        if (lane == 0) atomicOr(p.status, kStatusTimeout);
        // Copies in flight into this unit's ring (producer), then this
        // warp's MMAs.
        if (producer)
          for (int j = waited; j < issued; ++j)
            wait_w(bars + (j % depth) * 8, static_cast<uint32_t>((j / depth) & 1));
        if (lane == 0) tc_commit(drain + role * 8);
        __syncwarp();
        wait_w(drain + role * 8, 0u);
      }
    }
    ensure_waited();
    // Every warp of the CTA arrives here; the allocating warp frees TMEM.
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tbase, tc_cols);
    }
  } else {
  // ------------------------------------------------ mma.sync pipeline
  if (role == 0) {
    prepare_next();
    for (int i = 0; i < depth; ++i) {
      if (!issue(i)) {
        if constexpr (PAIR) send_end(i);
        break;
      }
      ++issued;
    }
  }

  // Accumulation in progress: head, segment, the head's segment range.
  int cur_head = -1, cur_slot = -1, cur_vfirst = 0, cur_vlast = 0;
  // The leader consumes the stages it issued; the follower runs until the
  // end record (every wait is bounded).
  for (int it = 0; role != 0 || it < issued; ++it) {
    const int slot = it % depth;
    const uint32_t par = static_cast<uint32_t>((it / depth) & 1);
    if (role != 0 && !mbar_wait(bars + slot * 8, par, kWaitLimitNs)) {
      ensure_waited();
      if (lane == 0) atomicOr(p.status, kStatusTimeout);
      return;  // the leader's copies are the leader's to wait for
    }
    const int4 m0 = meta[slot * 2];
    const int4 m1 = meta[slot * 2 + 1];
    if (PAIR && m0.x < 0) break;  // end record (follower)
    if (m0.x != cur_head || m1.x != cur_slot) {
      if (cur_head >= 0) finish_head(cur_head, cur_slot, cur_vfirst, cur_vlast);
      const bool new_head = m0.x != cur_head;
      cur_head = m0.x;
      cur_slot = m1.x;
      cur_vfirst = m1.z;
      cur_vlast = m1.w;
      start_head(cur_head, new_head);
    }
    if (role == 0 && !mbar_wait(bars + slot * 8, par, kWaitLimitNs)) {
      ensure_waited();
      if (lane == 0) atomicOr(p.status, kStatusTimeout);
      for (int j = it + 1; j < issued; ++j)
        mbar_wait(bars + (j % depth) * 8, static_cast<uint32_t>((j / depth) & 1),
                  kWaitLimitNs);
      return;
    }
    const int ntok_stage = m0.z << log2_bs;
    const int ntok_left = m0.w - (m0.y << log2_bs);
    const int ntok = ntok_stage < ntok_left ? ntok_stage : ntok_left;
    const int mtv = (ntok + 15) >> 4;
    const uint32_t kbase = ring + slot * STAGE_BYTES;
    const uint32_t vbase = kbase + KV_BYTES;
    bool dirty = false;
    if constexpr (CORE) {
      // q.K on CUDA cores: lane t scores token t against every query head.
      float sc[kCoreMaxG];
#pragma unroll
      for (int g = 0; g < kCoreMaxG; ++g) sc[g] = 0.f;
#pragma unroll
      for (int ch = 0; ch < D / 8; ++ch) {
        const uint4 kv = ld_shared_v4(kbase + (ch >> 3) * PLANE + lane * 128 +
                                      static_cast<uint32_t>(((ch & 7) ^ x7) << 4));
        float kf[8];
        unpack8<T>(kv, kf);
#pragma unroll
        for (int g = 0; g < kCoreMaxG; ++g) {
          if (g >= G) break;
          const float4 qa = *reinterpret_cast<const float4*>(qsm + g * D + ch * 8);
          const float4 qc = *reinterpret_cast<const float4*>(qsm + g * D + ch * 8 + 4);
          sc[g] = fmaf(qa.x, kf[0], sc[g]);
          sc[g] = fmaf(qa.y, kf[1], sc[g]);
          sc[g] = fmaf(qa.z, kf[2], sc[g]);
          sc[g] = fmaf(qa.w, kf[3], sc[g]);
          sc[g] = fmaf(qc.x, kf[4], sc[g]);
          sc[g] = fmaf(qc.y, kf[5], sc[g]);
          sc[g] = fmaf(qc.z, kf[6], sc[g]);
          sc[g] = fmaf(qc.w, kf[7], sc[g]);
        }
      }
      // Online softmax across the warp (tokens are lanes); rows past the
      // valid range are masked by selection, so stale shared memory never
      // reaches an arithmetic result.
      float pr[kCoreMaxG];
#pragma unroll
      for (int g = 0; g < kCoreMaxG; ++g) {
        if (g >= G) break;
        const float t = lane < ntok ? sc[g] * scale_log2 : -INFINITY;
        float mx = t;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mnew = fmaxf(cm[g], mx);
        const float alpha = fast_exp2(cm[g] - mnew);
        cm[g] = mnew;
        pr[g] = fast_exp2(t - mnew);
        cl[g] = cl[g] * alpha + pr[g];
        if (alpha != 1.f) {  // warp-uniform: the running max grew
#pragma unroll
          for (int e = 0; e < DL; ++e) cacc[g][e] *= alpha;
        }
      }
      // P.V: lane owns DL consecutive head-dim elements; p of token tt comes
      // from lane tt.  Only the ntok valid rows are read.
      const int hf = (lane * DL) >> 6;
      const int cidx = ((lane * DL) & 63) >> 3;
      const uint32_t boff = static_cast<uint32_t>(((lane * DL) & 7) * 2);
      for (int tt = 0; tt < ntok; ++tt) {
        const uint32_t addr = vbase + hf * PLANE + tt * 128 +
                              static_cast<uint32_t>((cidx ^ (tt & 7)) << 4) + boff;
        float vf[DL];
        load_row_part<T, DL>(addr, vf);
#pragma unroll
        for (int g = 0; g < kCoreMaxG; ++g) {
          if (g >= G) break;
          const float pt = __shfl_sync(0xffffffffu, pr[g], tt);
#pragma unroll
          for (int e = 0; e < DL; ++e) cacc[g][e] = fmaf(pt, vf[e], cacc[g][e]);
        }
      }
    } else {
    // S^T = K Q^T for the valid 16-token tiles; even and odd k-steps go to
    // separate accumulators so the two MMA dependency chains overlap.
    float sc[MT][NT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float s2[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sc[mt][nt][i] = 0.f;
          s2[nt][i] = 0.f;
        }
      if (mt < mtv) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t a[4];
          const int c = (ks & 3) * 2 + k_chunk;
          ldmatrix_x4(a, kbase + (ks >> 2) * PLANE + mt * 16 * 128 + k_lane +
                             static_cast<uint32_t>((c ^ x7) << 4));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (ks & 1)
              mma_16816<T>(s2[nt], a, qb[ks][nt][0], qb[ks][nt][1]);
            else
              mma_16816<T>(sc[mt][nt], a, qb[ks][nt][0], qb[ks][nt][1]);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[mt][nt][i] += s2[nt][i];
    }
    // Scale into log2 units; mask tokens past the valid range (tail only).
    if (ntok == ST) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) sc[mt][nt][i] *= scale_log2;
    } else {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int row = mt * 16 + lr + (i >> 1) * 8;
            sc[mt][nt][i] = row < ntok ? sc[mt][nt][i] * scale_log2 : -INFINITY;
          }
    }
    // Online softmax per query head (fragment column).
    float alpha[NT][2];
    bool grew = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float mx = -INFINITY;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) mx = fmaxf(mx, fmaxf(sc[mt][nt][e], sc[mt][nt][e + 2]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mold = mrun[nt][e];
        const float mnew = fmaxf(mold, mx);
        grew |= mnew > mold;
        alpha[nt][e] = fast_exp2(mold - mnew);
        mrun[nt][e] = mnew;
        float ls = 0.f;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const float p0 = fast_exp2(sc[mt][nt][e] - mnew);
          const float p2 = fast_exp2(sc[mt][nt][e + 2] - mnew);
          sc[mt][nt][e] = p0;
          sc[mt][nt][e + 2] = p2;
          ls += p0 + p2;
        }
        lrun[nt][e] = lrun[nt][e] * alpha[nt][e] + ls;
      }
    // Rescale the accumulator only when some running max grew.
    if (__any_sync(0xffffffffu, grew)) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int dt = 0; dt < KS; ++dt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[dt][nt][i] *= alpha[nt][i & 1];
    }
    // P^T fragments (B operand of the PV product) by in-register transpose.
    uint32_t pb[MT][NT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        pb[mt][nt][0] = 0u;
        pb[mt][nt][1] = 0u;
        if (mt < mtv) {
          pb[mt][nt][0] = movmatrix_trans(pack2<T>(sc[mt][nt][0], sc[mt][nt][1]));
          pb[mt][nt][1] = movmatrix_trans(pack2<T>(sc[mt][nt][2], sc[mt][nt][3]));
        }
      }
    // V rows past the valid range may hold stale or non-finite data; zero
    // them so 0 * V stays 0.  (Whole 128-byte rows: swizzle-invariant.)
    dirty = ntok < mtv * 16;
    if (dirty) {
      const int nrows = mtv * 16 - ntok;
      uint4* vz = reinterpret_cast<uint4*>(smem + (vbase - smem_base));
      for (int idx = lane; idx < nrows * NH * 8; idx += 32) {
        const int r = ntok + (idx >> (LOG2_NH + 3));
        const int hf = (idx >> 3) & (NH - 1), ch = idx & 7;
        vz[(hf * PLANE + r * 128) / 16 + ch] = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    // O^T += V^T P^T.
#pragma unroll
    for (int dt = 0; dt < KS; ++dt)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (mt < mtv) {
          uint32_t a[4];
          const int c = (dt & 3) * 2 + v_chunk;
          ldmatrix_x4_trans(a, vbase + (dt >> 2) * PLANE + mt * 16 * 128 + v_lane +
                                   static_cast<uint32_t>((c ^ x7) << 4));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_16816<T>(acc[dt][nt], a, pb[mt][nt][0], pb[mt][nt][1]);
        }
      }
    }  // MMA path
    __syncwarp();
    if (dirty) {
      fence_proxy_async_smem();
      __syncwarp();
    }
    if constexpr (PAIR) {
      if (role != 0) {  // the follower is done with the slot
        if (lane == 0) mbar_arrive(empties + slot * 8);
        continue;
      }
      if (sent_end) continue;
      // Refill only once the follower has released the slot (stage it).
      if (!mbar_wait(empties + slot * 8, par, kWaitLimitNs)) {
        ensure_waited();
        if (lane == 0) atomicOr(p.status, kStatusTimeout);
        for (int j = it + 1; j < issued; ++j)
          mbar_wait(bars + (j % depth) * 8, static_cast<uint32_t>((j / depth) & 1),
                    kWaitLimitNs);
        return;
      }
      if (issue(slot))
        ++issued;
      else
        send_end(slot);
    } else {
      if (issue(slot)) ++issued;
    }
  }
  if (cur_head >= 0) finish_head(cur_head, cur_slot, cur_vfirst, cur_vlast);
  ensure_waited();
  }  // pipelines
}


// Prologue of every reduce kernel: lets the next call's planner start (it
// writes nothing, the parity included, before this grid has finished),
// waits for the decode grid's partial states, then reads the current call's
// parity.
__device__ __forceinline__ uint32_t reduce_prologue(const DecodeParams& p) {
  grid_launch_dependents();
  grid_dependency_wait();  // partials written by the decode grid
  return *reinterpret_cast<volatile uint32_t*>(p.parity) & 1u;
}

// Segment range of head hd for the call with parity par.
__device__ __forceinline__ int2 head_segments(const DecodeParams& p, int hd, uint32_t par) {
  const int4 h = p.hseg[hd];
  return par ? make_int2(h.z, h.w) : make_int2(h.x, h.y);
}

// --------------------------------------------------------------------------
// Reduce kernels (the reduce of src/kernel_triton.py:120-174, planned on the
// device).  Row r = (head r / G, query head r % G) of a head whose pages fall
// in more than one segment folds the head's partial states, slots
// hd + hseg.x .. hd + hseg.x + hseg.y - 1, in slot order.
//
// reduce_heads_kernel: one warp per head, lanes over the head's G x D
// outputs (float4 f = lane + 32 k, k < NCT; query head g = 4 f / D), so each
// partial state is read once, coalesced; SB = 16 / NCT partials' loads are
// in flight per step.  For heads with few partials.  4 warps per CTA.
template <typename T, int D, int NCT>
__global__ void __launch_bounds__(128) reduce_heads_kernel(const DecodeParams p) {
  constexpr int SB = NCT >= 16 ? 1 : 16 / NCT;
  const int lane = threadIdx.x & 31;
  const int G = p.G, GD = G * D, nf = GD / 4;
  const int n_heads = p.B * p.Hkv;
  const int hd = blockIdx.x * 4 + (threadIdx.x >> 5);
  const uint32_t par = reduce_prologue(p);
  if (hd >= n_heads) return;
  const int2 hs = head_segments(p, hd, par);
  if (hs.y <= 1) return;  // empty, or written whole by the decode kernel
  const int sf = p.slot_floats;
  const float* base = p.part + static_cast<int64_t>(hd + hs.x) * sf;
  int gk[NCT];
  float M[NCT], L[NCT];
  float4 acc[NCT];
#pragma unroll
  for (int k = 0; k < NCT; ++k) {
    const int f = lane + 32 * k;
    gk[k] = f < nf ? (4 * f) / D : 0;
    M[k] = -INFINITY;
    L[k] = 0.f;
    acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int j0 = 0; j0 < hs.y; j0 += SB) {
    float4 v[SB][NCT];
    float mj[SB][NCT], lj[SB][NCT];
#pragma unroll
    for (int u = 0; u < SB; ++u) {
      const int j = j0 + u < hs.y ? j0 + u : hs.y - 1;
      const float* ps = base + static_cast<int64_t>(j) * sf;
#pragma unroll
      for (int k = 0; k < NCT; ++k) {
        const int f = lane + 32 * k;
        v[u][k] = f < nf ? __ldcg(reinterpret_cast<const float4*>(ps) + f) : make_float4(0.f, 0.f, 0.f, 0.f);
        mj[u][k] = __ldcg(ps + GD + gk[k]);
        lj[u][k] = __ldcg(ps + GD + G + gk[k]);
      }
    }
#pragma unroll
    for (int u = 0; u < SB; ++u) {
      if (j0 + u >= hs.y) break;
#pragma unroll
      for (int k = 0; k < NCT; ++k) {
        const float mn = fmaxf(M[k], mj[u][k]);
        const float sa = fast_exp2(M[k] - mn), sb = fast_exp2(mj[u][k] - mn);
        acc[k].x = acc[k].x * sa + v[u][k].x * sb;
        acc[k].y = acc[k].y * sa + v[u][k].y * sb;
        acc[k].z = acc[k].z * sa + v[u][k].z * sb;
        acc[k].w = acc[k].w * sa + v[u][k].w * sb;
        L[k] = L[k] * sa + lj[u][k] * sb;
        M[k] = mn;
      }
    }
  }
  const int Hq = p.Hkv * G;
  const int s = hd / p.Hkv, h = hd - s * p.Hkv;
#pragma unroll
  for (int k = 0; k < NCT; ++k) {
    const int f = lane + 32 * k;
    if (f >= nf) continue;
    const int g = gk[k], d = 4 * f - g * D;
    const int qh = h * G + g;
    const float inv = 1.f / L[k];
    if (p.state_o) {
      *reinterpret_cast<float4*>(p.state_o + (static_cast<int64_t>(s) * Hq + qh) * D + d) =
          make_float4(acc[k].x * inv, acc[k].y * inv, acc[k].z * inv, acc[k].w * inv);
      if (d == 0) p.state_lse[static_cast<int64_t>(s) * Hq + qh] = (M[k] + __log2f(L[k])) * kLn2;
    } else {
      T* o = static_cast<T*>(p.out) + s * p.o_sb + qh * p.o_sh + d;
      *reinterpret_cast<uint2*>(o) = make_uint2(pack2<T>(acc[k].x * inv, acc[k].y * inv),
                                                pack2<T>(acc[k].z * inv, acc[k].w * inv));
    }
  }
}

// reduce_rows_kernel: one warp per (head, query head) row — at D = 64 one
// half-warp per row, since a row is 16 float4 chunks — 16 partials' loads in
// flight per step; for large query groups (G * D > 1024) whose heads hold
// few partials.  4 warps per CTA.
template <typename T, int D>
__global__ void __launch_bounds__(128) reduce_rows_kernel(const DecodeParams p) {
  constexpr int RPW = D < 128 ? 128 / D : 1;  // rows per warp
  const int lane = threadIdx.x & 31;
  const int sub = lane % (32 / RPW);          // lane within the row's lanes
  const int G = p.G;
  const int rows = p.B * p.Hkv * G;
  const int r = (blockIdx.x * 4 + (threadIdx.x >> 5)) * RPW + lane / (32 / RPW);
  const uint32_t par = reduce_prologue(p);
  if (r >= rows) return;
  const int hd = r / G, g = r - hd * G;
  const int2 hs = head_segments(p, hd, par);
  if (hs.y <= 1) return;  // empty, or written whole by the decode kernel
  const float* bs1[1] = {p.part + static_cast<int64_t>(hd + hs.x) * p.slot_floats};
  const int g1[1] = {g}, a1[1] = {0}, b1[1] = {hs.y};
  float M[1], L[1];
  float4 acc[1][(D + 127) / 128];
  fold_rows<D, 1, 16>(bs1, g1, a1, b1, p.slot_floats, G, sub, M, L, acc);
  write_row<T, D>(p, hd, g, sub, M[0], L[0], acc[0]);
}

// reduce_split_kernel: one CTA of 4 warps per row; warp w folds partials
// [w n / 4, (w + 1) n / 4) and the 4 states are combined in order through
// shared memory; for heads with many partials.
template <typename T, int D>
__global__ void __launch_bounds__(128) reduce_split_kernel(const DecodeParams p) {
  // rows padded to D + 4 floats: every row starts on a 16-byte boundary for
  // the float4 accesses below; [D] holds M, [D + 1] holds L
  __shared__ __align__(16) float part_sm[4][D + 4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G;
  const int r = blockIdx.x;
  const uint32_t par = reduce_prologue(p);
  const int hd = r / G, g = r - hd * G;
  const int2 hs = head_segments(p, hd, par);
  if (hs.y <= 1) return;  // uniform across the CTA
  constexpr int NC = (D + 127) / 128;
  const int a = static_cast<int>(static_cast<int64_t>(warp) * hs.y / 4);
  const int b = static_cast<int>(static_cast<int64_t>(warp + 1) * hs.y / 4);
  float M[1] = {-INFINITY}, L[1] = {0.f};
  float4 acc[1][NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) acc[0][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (b > a) {
    const float* bs1[1] = {p.part + static_cast<int64_t>(hd + hs.x) * p.slot_floats};
    const int g1[1] = {g}, a1[1] = {a}, b1[1] = {b};
    fold_rows<D, 1, 16>(bs1, g1, a1, b1, p.slot_floats, G, lane, M, L, acc);
  }
#pragma unroll
  for (int c = 0; c < NC; ++c)
    if (lane * 4 + 128 * c < D) *reinterpret_cast<float4*>(&part_sm[warp][lane * 4 + 128 * c]) = acc[0][c];
  if (lane == 0) {
    part_sm[warp][D] = M[0];
    part_sm[warp][D + 1] = L[0];
  }
  __syncthreads();
  if (warp != 0) return;
  float Mx = -INFINITY, Lx = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) Mx = fmaxf(Mx, part_sm[q][D]);
  float4 o[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) o[c] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float sc = fast_exp2(part_sm[q][D] - Mx);  // an empty part: 2^-inf = 0
    Lx += sc * part_sm[q][D + 1];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int cc = lane * 4 + 128 * c;
      if (cc >= D) continue;
      const float4 x = *reinterpret_cast<const float4*>(&part_sm[q][cc]);
      o[c].x += sc * x.x;
      o[c].y += sc * x.y;
      o[c].z += sc * x.z;
      o[c].w += sc * x.w;
    }
  }
  write_row<T, D>(p, hd, g, lane, Mx, Lx, o);
}

// --------------------------------------------------------------------------
// Cross-device merge of (o, lse) states: one warp per output row.
template <typename TO>
__device__ __forceinline__ void store_out4(TO* o, float4 v);
template <>
__device__ __forceinline__ void store_out4<float>(float* o, float4 v) {
  *reinterpret_cast<float4*>(o) = v;
}
template <>
__device__ __forceinline__ void store_out4<__nv_bfloat16>(__nv_bfloat16* o, float4 v) {
  *reinterpret_cast<uint2*>(o) = make_uint2(pack2<__nv_bfloat16>(v.x, v.y), pack2<__nv_bfloat16>(v.z, v.w));
}
template <>
__device__ __forceinline__ void store_out4<__half>(__half* o, float4 v) {
  *reinterpret_cast<uint2*>(o) = make_uint2(pack2<__half>(v.x, v.y), pack2<__half>(v.z, v.w));
}

template <typename TO>
__global__ void __launch_bounds__(256) merge_states_kernel(
    const float* __restrict__ so, int64_t o_stride, const float* __restrict__ slse,
    int64_t lse_stride, int n, int64_t rows, int D, TO* __restrict__ out,
    int64_t out_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float M = -INFINITY;
  for (int i = 0; i < n; ++i) M = fmaxf(M, slse[i * lse_stride + row]);
  for (int c = lane * 4; c < D; c += 128) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    float L = 0.f;
    if (M != -INFINITY) {
      for (int i = 0; i < n; ++i) {
        const float w = fast_exp2((slse[i * lse_stride + row] - M) * kLog2e);
        const float4 v = *reinterpret_cast<const float4*>(so + i * o_stride + row * D + c);
        a.x += w * v.x;
        a.y += w * v.y;
        a.z += w * v.z;
        a.w += w * v.w;
        L += w;
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    store_out4<TO>(out + row * out_stride + c, make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv));
  }
}

// --------------------------------------------------------------------------
// KV append (the step before a decode; no counterpart in the reference).
// One warp per sequence.  Lane h (per group of 32 kv heads) reads head h's
// current length L and its page id together, so every head's length is read
// before any changes; the new K and V rows (head_size 2-byte elements copied
// as 32-bit words, lanes over the words) are then copied four heads at a
// time with their loads in flight together, into row L % bs of page
// block_table[L / bs]; last, the lengths move.  A length shared by all heads
// of a sequence (h stride 0) moves once, if every head's token was written.

__global__ void __launch_bounds__(128) kv_append_kernel(const AppendParams p) {
  const int lane = threadIdx.x & 31;
  const int s = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (s >= p.B) return;
  const int words = p.D / 2;
  const int hc_rows = p.head_in_page ? p.Hkv : 1;
  uint32_t flags = 0;
  bool all_ok = true;
  for (int h0 = 0; h0 < p.Hkv; h0 += 32) {
    // lane h: head h0 + h's length, page and destination row
    const int h = h0 + lane;
    int L = -1;
    bool ok = false;
    int64_t row = 0;
    if (h < p.Hkv) {
      L = p.lens[s * p.l_sb + h * p.l_sh];
      ok = L >= 0;
      if (ok && L / p.bs >= p.maxb) {
        flags |= kStatusAppendFull;
        ok = false;
      }
      if (ok) {
        const int64_t pid =
            static_cast<int64_t>(p.bt[s * p.bt_sb + h * p.bt_sh + static_cast<int64_t>(L / p.bs) * p.bt_si]) *
                p.bt_mul + static_cast<int64_t>(h) * p.bt_add;
        if (pid < 0 || pid >= p.num_pages) {
          flags |= kStatusBadPage;
          ok = false;
        }
        row = (pid * p.bs + L % p.bs) * hc_rows + (p.head_in_page ? h : 0);
      }
    }
    all_ok &= __all_sync(0xffffffffu, ok || h >= p.Hkv);
    const int nh = min(32, p.Hkv - h0);
    for (int c0 = 0; c0 < nh; c0 += 4) {
      uint32_t kw[4][4], vw[4][4];  // 4 heads x up to 4 words per lane (head_size <= 256)
      bool hok[4];
      int64_t hrow[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u < nh ? c0 + u : nh - 1;
        hok[u] = __shfl_sync(0xffffffffu, ok, c) && c0 + u < nh;
        hrow[u] = __shfl_sync(0xffffffffu, row, c);
        const int64_t src = (s * p.n_sb + static_cast<int64_t>(h0 + c) * p.n_sh) / 2;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int w = lane + 32 * q;
          kw[u][q] = hok[u] && w < words ? p.k_new[src + w] : 0u;
          vw[u][q] = hok[u] && w < words ? p.v_new[src + w] : 0u;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (!hok[u]) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int w = lane + 32 * q;
          if (w < words) {
            p.k_cache[hrow[u] * words + w] = kw[u][q];
            p.v_cache[hrow[u] * words + w] = vw[u][q];
          }
        }
      }
    }
    if (p.increment && p.l_sh != 0 && ok) p.lens[s * p.l_sb + h * p.l_sh] = L + 1;
  }
  if (p.increment && p.l_sh == 0 && all_ok && lane == 0) p.lens[s * p.l_sb] += 1;
  flags = __reduce_or_sync(0xffffffffu, flags);
  if (flags && lane == 0 && p.status) atomicOr(p.status, flags);
}

// --------------------------------------------------------------------------
// Fused exchange + merge of partial states over peer memory (ranks of one
// node, buffers mapped with CUDA IPC).  Replaces all-gather + merge_states for
// a context split across GPUs.
//
// Every value crosses NVLink as one 64-bit word {float bits, epoch}, stored
// and loaded with relaxed system-scope accesses (single-copy atomic), so a
// reader that sees the current epoch in a word also sees its value: no fence,
// no separate flag and no second NVLink trip.  Block b of every rank owns the
// same rows [r0, r1): it stores this rank's o and lse of those rows into slot
// [parity][rank] of every peer's buffer, then merges the rows, waiting
// (bounded) for each peer word of the current epoch in its own memory.
//
// Exchange buffer of each rank: [2][world][S] uint64 words, then uint32
// epoch[nb] (calls block b has made; nb = exchange_blocks(rows), the same on
// every rank).  The two parities let a peer run one call ahead while this
// rank still reads the previous call's slots; a peer cannot get two calls
// ahead because its next call waits for this rank's words of the call in
// between, which this rank stores only after finishing the current one.
struct ExchangeParams {
  float* state;             // this rank's packed state: o [rows, D], lse [rows]
  uint64_t* const* bufs;    // [world] exchange buffers as mapped here (bufs[rank] own)
  int32_t rank, world;
  int64_t S;                // floats per packed state (multiple of 4)
  int64_t rows;
  int32_t D;
  int64_t rows_per_block;
  void* out;
  int64_t out_stride;
  uint64_t wait_limit_ns;
  uint32_t* status;         // PAB200_STATUS_* bits (timeout)
  // Fused with the decode call that wrote `state` (part != nullptr): the
  // rows of heads that call split over several segments are still partial
  // states in its workspace; each block first folds its own rows' partials
  // into `state` (the reduce kernel's merge, in this kernel), then exchanges.
  // Row r is query head r % G of head r / G.
  const float* part;
  const int4* hseg;
  const uint32_t* parity;
  int32_t slot_floats;
  int32_t G;
};

// One block per row up to 1024 rows (a block's warps then split the row's
// partial states between them), a few rows per block beyond.
__host__ __device__ inline int64_t exchange_blocks(int64_t rows) {
  return rows < 1 ? 1 : (rows < 1024 ? rows : 1024);
}

__device__ __forceinline__ uint64_t ll_word(float v, uint32_t e) {
  return (static_cast<uint64_t>(e) << 32) | __float_as_uint(v);
}

// Loads N words at p[0], p[step], ... once all carry epoch e.  On timeout
// sets the status bit, stops waiting for the rest of this thread's loads
// (`gave_up`) and returns what is there.
template <int N>
__device__ __forceinline__ void ll_load(const uint64_t* p, int64_t step, uint32_t e, float* v,
                                        bool& gave_up, const ExchangeParams& prm) {
  uint64_t w[N];
  bool ready = true;
#pragma unroll
  for (int k = 0; k < N; ++k) {
    w[k] = ld_relaxed_sys_u64(p + k * step);
    ready &= static_cast<uint32_t>(w[k] >> 32) == e;
  }
  if (!ready && !gave_up) {
    const uint64_t t0 = global_timer_ns();
    while (!ready) {
      ready = true;
#pragma unroll
      for (int k = 0; k < N; ++k) {
        if (static_cast<uint32_t>(w[k] >> 32) != e) w[k] = ld_relaxed_sys_u64(p + k * step);
        ready &= static_cast<uint32_t>(w[k] >> 32) == e;
      }
      if (!ready && global_timer_ns() - t0 > prm.wait_limit_ns) {
        atomicOr(prm.status, kStatusTimeout);
        gave_up = true;
        break;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < N; ++k) v[k] = __uint_as_float(static_cast<uint32_t>(w[k]));
}

template <typename TO, int DF>
__global__ void __launch_bounds__(256) exchange_merge_kernel(const ExchangeParams p) {
  const int world = p.world, rank = p.rank;
  const int64_t S = p.S, rows = p.rows;
  const int D = p.D;
  const int tid = threadIdx.x, b = blockIdx.x;
  const int64_t r0 = b * p.rows_per_block;
  const int64_t r1 = r0 + p.rows_per_block < rows ? r0 + p.rows_per_block : rows;
  uint32_t* epochs = reinterpret_cast<uint32_t*>(p.bufs[rank] + 2 * world * S);
  // The next call's planner may start at once: it writes nothing before
  // this grid has finished.  `state` (and, after a previous exchange,
  // `epochs`) were written by the preceding grid on this stream: read them
  // only after it has completed.
  grid_launch_dependents();
  grid_dependency_wait();
  if constexpr (DF > 0) {
    // 0. fused with the decode call: fold the split heads' partial states of
    //    rows [r0, r1) into `state` in slot order (the reduce kernels'
    //    merge), one warp per row; rows of whole or empty heads were written
    //    by the decode grid already.  With fewer rows than warps the warps
    //    of a row split its partials into contiguous parts and the row's
    //    first warp combines the parts in order (so the result depends
    //    only on the segment count, not on timing).
    if (p.part) {
      constexpr int NC = (DF + 127) / 128;
      __shared__ float4 sacc[8][32][NC];
      __shared__ float sml[8][2];
      const int warp = tid >> 5, lane = tid & 31;
      const int nw = blockDim.x >> 5;  // 8
      const int rpb = static_cast<int>(r1 - r0);
      int wpr = 1;  // warps per row
      while (wpr < nw && wpr * 2 * rpb <= nw) wpr *= 2;
      const int rows_per_round = nw / wpr;
      const int sub = warp % wpr;
      const uint32_t hpar = *reinterpret_cast<const volatile uint32_t*>(p.parity) & 1u;
      for (int64_t base = r0; base < r1; base += rows_per_round) {
        const int64_t row = base + warp / wpr;
        int hd = 0, g = 0;
        int2 hs = make_int2(0, 0);
        if (row < r1) {
          hd = static_cast<int>(row / p.G);
          g = static_cast<int>(row - int64_t(hd) * p.G);
          const int4 h4 = p.hseg[hd];
          hs = hpar ? make_int2(h4.z, h4.w) : make_int2(h4.x, h4.y);
        }
        const bool split = row < r1 && hs.y > 1;
        float M[1] = {-INFINITY}, L[1] = {0.f};
        float4 acc[1][NC];
#pragma unroll
        for (int i = 0; i < NC; ++i) acc[0][i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (split) {
          const float* bs1[1] = {p.part + static_cast<int64_t>(hd + hs.x) * p.slot_floats};
          const int g1[1] = {g};
          const int a1[1] = {sub * hs.y / wpr}, b1[1] = {(sub + 1) * hs.y / wpr};
          fold_rows<DF, 1, 16>(bs1, g1, a1, b1, p.slot_floats, p.G, lane, M, L, acc);
        }
        if (wpr > 1) {
          if (lane == 0) {
            sml[warp][0] = M[0];
            sml[warp][1] = L[0];
          }
#pragma unroll
          for (int i = 0; i < NC; ++i) sacc[warp][lane][i] = acc[0][i];
          __syncthreads();
          if (split && sub == 0) {
            for (int w = warp + 1; w < warp + wpr; ++w) {
              const float mw = sml[w][0];
              if (mw == -INFINITY) continue;  // an empty part
              const float mn = fmaxf(M[0], mw);
              const float sa = M[0] == -INFINITY ? 0.f : fast_exp2(M[0] - mn);
              const float sb = fast_exp2(mw - mn);
#pragma unroll
              for (int i = 0; i < NC; ++i) {
                const float4 v = sacc[w][lane][i];
                acc[0][i].x = acc[0][i].x * sa + v.x * sb;
                acc[0][i].y = acc[0][i].y * sa + v.y * sb;
                acc[0][i].z = acc[0][i].z * sa + v.z * sb;
                acc[0][i].w = acc[0][i].w * sa + v.w * sb;
              }
              L[0] = L[0] * sa + sml[w][1] * sb;
              M[0] = mn;
            }
          }
          __syncthreads();  // sacc / sml are reused by the next round
        }
        if (split && sub == 0) {
          const float inv = 1.f / L[0];
#pragma unroll
          for (int i = 0; i < NC; ++i) {
            const int c = lane * 4 + 128 * i;
            if (c < DF)
              *reinterpret_cast<float4*>(p.state + row * DF + c) =
                  make_float4(acc[0][i].x * inv, acc[0][i].y * inv, acc[0][i].z * inv,
                              acc[0][i].w * inv);
          }
          if (lane == 0) p.state[rows * DF + row] = (M[0] + __log2f(L[0])) * kLn2;
        }
      }
      __syncthreads();  // the block's rows are final before they are sent
    }
  }
  const uint32_t e = reinterpret_cast<volatile uint32_t*>(epochs)[b] + 1u;
  const int par = e & 1;
  // 1. store rows [r0, r1) of o and lse into every peer's slot [par][rank]
  const float* st = p.state;
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    uint64_t* slot = p.bufs[r] + (static_cast<int64_t>(par) * world + rank) * S;
    for (int64_t i = r0 * D + 2 * tid; i < r1 * D; i += 2 * blockDim.x) {
      const float2 v = *reinterpret_cast<const float2*>(st + i);
      st_relaxed_sys_u64(slot + i, ll_word(v.x, e));
      st_relaxed_sys_u64(slot + i + 1, ll_word(v.y, e));
    }
    for (int64_t i = rows * D + r0 + tid; i < rows * D + r1; i += blockDim.x)
      st_relaxed_sys_u64(slot + i, ll_word(st[i], e));
  }
  if (tid == 0) epochs[b] = e;  // read only by this block's next call
  // 2. merge rows [r0, r1): one warp per row, lanes over the head dimension;
  //    slot i holds rank i's words, this rank's own state is read directly
  const int lane = tid & 31;
  const uint64_t* slots = p.bufs[rank] + static_cast<int64_t>(par) * world * S;
  bool gave_up = false;
  for (int64_t row = r0 + (tid >> 5); row < r1; row += blockDim.x / 32) {
    float M = -INFINITY;
    for (int i = 0; i < world; ++i) {
      float l;
      if (i == rank) l = st[rows * D + row];
      else ll_load<1>(slots + i * S + rows * D + row, 1, e, &l, gave_up, p);
      M = fmaxf(M, l);
    }
    for (int c = lane * 4; c < D; c += 128) {
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      float L = 0.f;
      if (M != -INFINITY) {
        for (int i = 0; i < world; ++i) {
          float l, v[4];
          if (i == rank) {
            l = st[rows * D + row];
            const float4 o = *reinterpret_cast<const float4*>(st + row * D + c);
            v[0] = o.x, v[1] = o.y, v[2] = o.z, v[3] = o.w;
          } else {
            ll_load<1>(slots + i * S + rows * D + row, 1, e, &l, gave_up, p);
            ll_load<4>(slots + i * S + row * D + c, 1, e, v, gave_up, p);
          }
          const float w = fast_exp2((l - M) * kLog2e);
          a.x += w * v[0];
          a.y += w * v[1];
          a.z += w * v[2];
          a.w += w * v[3];
          L += w;
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      store_out4<TO>(static_cast<TO*>(p.out) + row * p.out_stride + c,
                     make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv));
    }
  }
}

}  // namespace pab

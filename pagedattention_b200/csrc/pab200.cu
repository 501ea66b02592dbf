// libpab200.so — host side of the C ABI declared in include/pab200.h.
//
// Replaces the host wrapper flash_attn_with_kvcache_wrapper_triton
// (src/kernel_triton.py:181-307).  Differences by design: the chunk plan is
// computed on the device (no .cpu() sync, no per-call H2D metadata copies,
// src/kernel_triton.py:206-229), the partial buffers live in a caller-owned
// workspace (no per-call allocation, :232-243), and the reduce kernel is
// scheduled while the decode grid runs (programmatic dependent launch).
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <mutex>

#include "decode.cuh"
#include "pab200.h"

#define PAB200_EXPORT extern "C" __attribute__((visibility("default")))

extern char** environ;  // the process environment (POSIX)

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PAB200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

constexpr int kMaxDevices = 64;

int device_sm_count(int dev) {
  static int sms[kMaxDevices] = {0};
  static std::mutex mu;
  if (dev < 0 || dev >= kMaxDevices) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      sms[dev] = n;
  }
  return sms[dev];
}

int device_sm_count_current() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  const int n = device_sm_count(dev);
  return n > 0 ? n : 148;
}

// Tuning variables (PAB200_*), read from the environment: one pass over
// the environment per planned call collects the (usually zero) PAB200_
// entries, so a call does not pay a full getenv scan per variable, and a
// variable changed between calls is seen by the next one.
struct EnvSnapshot {
  const char* entries[16];
  int n = 0;
};
thread_local EnvSnapshot g_env;

void refresh_env() {
  g_env.n = 0;
  for (char** e = environ; e && *e && g_env.n < 16; ++e)
    if (std::strncmp(*e, "PAB200_", 7) == 0) g_env.entries[g_env.n++] = *e;
}

int env_int(const char* name, int fallback) {
  const size_t len = std::strlen(name);
  for (int i = 0; i < g_env.n; ++i) {
    const char* e = g_env.entries[i];
    if (std::strncmp(e, name, len) == 0 && e[len] == '=')
      return e[len + 1] ? std::atoi(e + len + 1) : fallback;
  }
  return fallback;
}

// ------------------------------------------------------------------ kernels
struct KernelOps {
  void* fn;  // decode kernel (for attributes / occupancy)
  cudaError_t (*launch)(dim3, dim3, size_t, cudaStream_t, bool, const CUtensorMap&,
                        const CUtensorMap&, const pab::DecodeParams&);
};

// Launch configuration; `pdl` lets the grid start while the previous kernel
// in the stream finishes (programmatic dependent launch): the kernel waits
// with griddepcontrol.wait before it reads that kernel's output.
struct LaunchCfg {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  LaunchCfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl) {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
  }
};

template <typename T, int D, int NT, int ST, bool CORE, bool PAIR, bool TC>
cudaError_t launch_decode(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                          const CUtensorMap& k, const CUtensorMap& v,
                          const pab::DecodeParams& p) {
  LaunchCfg lc(grid, block, smem, s, pdl);
  return cudaLaunchKernelEx(&lc.cfg, pab::decode_kernel<T, D, NT, ST, CORE, PAIR, TC>, k, v, p);
}

template <typename T, int D, int NT, int ST, bool CORE = false, bool PAIR = false, bool TC = false>
KernelOps ops_of() {
  return KernelOps{reinterpret_cast<void*>(&pab::decode_kernel<T, D, NT, ST, CORE, PAIR, TC>),
                   &launch_decode<T, D, NT, ST, CORE, PAIR, TC>};
}

template <typename T, int ST>
bool select_dnt(int D, int nt, bool core, bool pair, bool tc, KernelOps* o) {
  if (tc) {  // tcgen05 path: D 64, 64-token stages, two warps per ring
    if (ST != 64 || D != 64 || !pair || nt != 2) return false;
    *o = ops_of<T, 64, 2, 64, false, true, true>();
    return true;
  }
  if (pair) {  // two warps per ring, 16 query heads each
    if (nt != 2) return false;
    switch (D) {
      case 64: *o = ops_of<T, 64, 2, ST, false, true>(); return true;
      case 128: *o = ops_of<T, 128, 2, ST, false, true>(); return true;
      default: return false;
    }
  }
  if (core) {  // CUDA-core path: G <= 4, 32-token stages, D <= 128
    if (ST != 32 || nt != 1) return false;
    switch (D) {
      case 64: *o = ops_of<T, 64, 1, 32, true>(); return true;
      case 128: *o = ops_of<T, 128, 1, 32, true>(); return true;
      default: return false;
    }
  }
  switch (D * 16 + nt) {
    case 64 * 16 + 1: *o = ops_of<T, 64, 1, ST>(); return true;
    case 64 * 16 + 2: *o = ops_of<T, 64, 2, ST>(); return true;
    case 64 * 16 + 4: *o = ops_of<T, 64, 4, ST>(); return true;
    case 128 * 16 + 1: *o = ops_of<T, 128, 1, ST>(); return true;
    case 128 * 16 + 2: *o = ops_of<T, 128, 2, ST>(); return true;
    case 256 * 16 + 1: *o = ops_of<T, 256, 1, ST>(); return true;
    default: return false;
  }
}

bool select_kernel(int dtype, int D, int nt, int st, bool core, bool pair, bool tc,
                   KernelOps* o) {
  if (dtype == PAB200_DTYPE_BF16) {
    switch (st) {
      case 16: return !tc && select_dnt<__nv_bfloat16, 16>(D, nt, core, pair, false, o);
      case 32: return !tc && select_dnt<__nv_bfloat16, 32>(D, nt, core, pair, false, o);
      case 64: return select_dnt<__nv_bfloat16, 64>(D, nt, core, pair, tc, o);
      default: return false;
    }
  }
  switch (st) {
    case 16: return !tc && select_dnt<__half, 16>(D, nt, core, pair, false, o);
    case 32: return !tc && select_dnt<__half, 32>(D, nt, core, pair, false, o);
    case 64: return select_dnt<__half, 64>(D, nt, core, pair, tc, o);
    default: return false;
  }
}

// ------------------------------------------------------------------ planning
struct Plan {
  KernelOps ops;
  int G, nt, st, wpc, depth, ctas_per_sm, grid, W;
  bool core, pair, tc;
  size_t smem;
  int n_heads;
  int slot_floats;
  int steal_m_max, steal_min_stages;
  size_t off_cum, off_wstart, off_claims, off_hseg, off_empty, off_part, ws_bytes;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// Checks shapes, sizes and (with check_pointers) pointers and alignment.
int validate(const pab200_decode_args* a, bool check_pointers) {
  if (!a) return fail(PAB200_ERR_INVALID_ARGUMENT, "args is null");
  if (a->dtype != PAB200_DTYPE_BF16 && a->dtype != PAB200_DTYPE_F16)
    return fail(PAB200_ERR_UNSUPPORTED, "dtype %d: q/k/v must be bf16 or f16", a->dtype);
  if (a->layout != PAB200_LAYOUT_PAGES && a->layout != PAB200_LAYOUT_NHD)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "unknown cache layout %d", a->layout);
  if (a->num_seqs < 1 || a->num_kv_heads < 1 || a->num_q_heads < 1)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "num_seqs, num_q_heads, num_kv_heads must be >= 1");
  if (a->num_q_heads % a->num_kv_heads != 0)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "num_q_heads (%d) %% num_kv_heads (%d) != 0",
                a->num_q_heads, a->num_kv_heads);
  const int D = a->head_size, bs = a->block_size;
  if (D != 64 && D != 128 && D != 256)
    return fail(PAB200_ERR_UNSUPPORTED, "head_size %d: supported 64, 128, 256", D);
  if (bs != 8 && bs != 16 && bs != 32 && bs != 64)
    return fail(PAB200_ERR_UNSUPPORTED, "block_size %d: supported 8, 16, 32, 64", bs);
  const int G = a->num_q_heads / a->num_kv_heads;
  // One warp holds at most 16 query heads x 128 (or 8 x 256) accumulators;
  // groups of 17-32 heads at D <= 128 are split over a pair of warps.
  if (G * D > 2048 && !(G <= 32 && D <= 128))
    return fail(PAB200_ERR_UNSUPPORTED,
                "query group %d x head_size %d exceeds the register tile "
                "(G*D <= 2048, or G <= 32 with head_size <= 128)", G, D);
  if (a->max_blocks < 0 || a->num_pages < 0)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "max_blocks and num_pages must be >= 0");
  const int64_t n_heads = int64_t(a->num_seqs) * a->num_kv_heads;
  if (n_heads * (a->max_blocks > 0 ? a->max_blocks : 1) >= (int64_t(1) << 31) ||
      int64_t(a->max_blocks) * bs >= (int64_t(1) << 31))
    return fail(PAB200_ERR_UNSUPPORTED, "num_seqs*num_kv_heads*max_blocks too large (>= 2^31)");
  if (a->num_pages * bs >= (int64_t(1) << 31))
    return fail(PAB200_ERR_UNSUPPORTED, "num_pages*block_size too large (>= 2^31 rows)");
  if (a->num_pages == 0 && a->max_blocks > 0)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "num_pages is 0 but max_blocks > 0");
  if (a->num_splits < 0) return fail(PAB200_ERR_INVALID_ARGUMENT, "num_splits must be >= 0");
  if (!check_pointers) return PAB200_OK;
  if (!a->q || !a->seqlens) return fail(PAB200_ERR_INVALID_ARGUMENT, "q or seqlens is null");
  if (!a->state_o && !a->out) return fail(PAB200_ERR_INVALID_ARGUMENT, "out is null");
  if (a->state_o && !a->state_lse)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "state_o given without state_lse");
  if (a->num_pages > 0 && (!a->k_cache || !a->v_cache || !a->block_table))
    return fail(PAB200_ERR_INVALID_ARGUMENT, "k_cache, v_cache or block_table is null");
  if (!aligned(a->q, 4) || (a->q_stride_b & 1) || (a->q_stride_h & 1))
    return fail(PAB200_ERR_ALIGNMENT, "q must be 4-byte aligned with even strides");
  if (!a->state_o && (!aligned(a->out, 8) || (a->out_stride_b & 3) || (a->out_stride_h & 3)))
    return fail(PAB200_ERR_ALIGNMENT, "out must be 8-byte aligned with strides that are multiples of 4");
  if (a->state_o && (!aligned(a->state_o, 16) || !aligned(a->state_lse, 4)))
    return fail(PAB200_ERR_ALIGNMENT, "state_o must be 16-byte aligned");
  if (a->num_pages > 0 && (!aligned(a->k_cache, 16) || !aligned(a->v_cache, 16)))
    return fail(PAB200_ERR_ALIGNMENT, "k_cache and v_cache must be 16-byte aligned");
  return PAB200_OK;
}

// Dynamic shared memory of one decode CTA: ring slots, (tcgen05 path) the
// query and probability tiles of every unit pair, then per-unit mbarriers,
// stage records and CUDA-core query scratch (see decode_kernel), then the
// early-start page-count prefix (single-warp rings).  A paired kernel has
// one ring (and a second set of mbarriers) per two warps; the tcgen05 path
// adds its own mbarriers and the tensor-memory address.
size_t decode_smem(int wpc, int depth, size_t stage, bool pair, int core_bytes, bool tc) {
  const size_t units = pair ? size_t(wpc / 2) : size_t(wpc);
  return 1024 + units * depth * stage +
         (tc ? (units + 1) / 2 * 2 * pab::kTcTileBytes : 0) +
         units * (pab::kMaxDepth * (8 + pab::kMetaBytesPerSlot) + core_bytes) +
         (pair ? units * pab::kMaxDepth * 8 : size_t(pab::kEarlyBytes)) +
         (tc ? units * pab::kTcBarsPerUnit * 8 + 16 : 0);
}

// Tensor-memory columns one CTA of the tcgen05 path allocates (a power of
// two; the kernel computes the same).
int tc_cols(int units) { return units > 2 ? 512 : units * pab::kTcUnitCols; }

struct Geometry {
  int wpc, per_sm;
  size_t smem;
};

// Warps per CTA and CTAs per SM for one decode kernel.  Each warp's stage
// loop is latency-bound, so throughput follows the number of resident warps:
// try every CTA size and keep the one with the most warps per SM (shared
// memory and registers both limit it; ties go to the larger CTA).  Results
// are cached per device, kernel, ring depth and stage size.
int choose_geometry(const KernelOps& ops, int dev, int depth, size_t stage, bool pair,
                    int core_bytes, bool tc, int forced_wpc, Geometry* out) {
  struct Entry {
    int dev;
    void* fn;
    int depth;
    size_t stage;
    int forced;
    Geometry g;
  };
  static Entry cache[128];
  static int used = 0;
  static void* attr_set[kMaxDevices][64] = {{nullptr}};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].dev == dev && cache[i].fn == ops.fn && cache[i].depth == depth &&
        cache[i].stage == stage && cache[i].forced == forced_wpc) {
      *out = cache[i].g;
      return PAB200_OK;
    }
  if (dev < 0 || dev >= kMaxDevices) return fail(PAB200_ERR_CUDA, "device index %d out of range", dev);
  bool have_attr = false;
  for (int i = 0; i < 64 && attr_set[dev][i]; ++i) have_attr |= attr_set[dev][i] == ops.fn;
  if (!have_attr) {
    cudaError_t e = cudaFuncSetAttribute(ops.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    for (int i = 0; i < 64; ++i)
      if (!attr_set[dev][i]) {
        attr_set[dev][i] = ops.fn;
        break;
      }
  }
  if (forced_wpc && (forced_wpc < 1 || forced_wpc > pab::kMaxWarpsPerCta))
    return fail(PAB200_ERR_INVALID_ARGUMENT, "PAB200_WPC must be in [1, %d]", pab::kMaxWarpsPerCta);
  static const int kCandidates[] = {8, 6, 4, 3, 2, 1};
  const int* cand = forced_wpc ? &forced_wpc : kCandidates;
  const int ncand = forced_wpc ? 1 : 6;
  Geometry best{0, 0, 0};
  for (int ci = 0; ci < ncand; ++ci) {
    const int wpc = cand[ci];
    if (pair && (wpc & 1)) continue;  // warps come in pairs
    const size_t smem = decode_smem(wpc, depth, stage, pair, core_bytes, tc);
    if (smem > 232448) continue;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ops.fn, wpc * 32, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    // tcgen05 path: the resident CTAs' tensor memory must fit the SM's 512
    // columns, so that no allocation waits for another CTA.
    if (tc) per_sm = std::min(per_sm, 512 / tc_cols(wpc / 2));
    if (per_sm * wpc > best.per_sm * best.wpc) best = Geometry{wpc, per_sm, smem};
  }
  if (best.per_sm < 1) return fail(PAB200_ERR_UNSUPPORTED, "decode kernel does not fit on an SM");
  if (used < 128) cache[used++] = Entry{dev, ops.fn, depth, stage, forced_wpc, best};
  *out = best;
  return PAB200_OK;
}

// Plans one call.  `scratch_cap`: largest workspace the call may use; the
// tail-chunk count per warp (m_max) is lowered until the workspace fits it
// (SIZE_MAX for a caller workspace, which is sized to the plan instead).
int make_plan(const pab200_decode_args* a, Plan* pl, size_t scratch_cap,
              bool check_pointers = true) {
  refresh_env();
  int rc = validate(a, check_pointers);
  if (rc) return rc;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const int sms = device_sm_count(dev);
  if (sms <= 0) return fail(PAB200_ERR_CUDA, "cannot query the SM count of device %d", dev);

  const int D = a->head_size, bs = a->block_size;
  pl->G = a->num_q_heads / a->num_kv_heads;
  pl->nt = pl->G <= 8 ? 1 : (pl->G <= 16 ? 2 : 4);
  // Groups of 17-32 query heads that one warp cannot hold (D = 128): two
  // warps share each ring, 16 heads each.  At D = 64 one warp holds all 32
  // and is faster (mqa_small_page: 54.4 against 64.9 us per call for the
  // pair), so pairs are used there only when PAB200_PAIR=1 asks for them.
  const bool pair_ok = pl->G > 16 && pl->G <= 32 && (D == 64 || D == 128);
  pl->pair = pair_ok && env_int("PAB200_PAIR", pl->G * D > 2048 ? 1 : 0) != 0;
  // tcgen05 path (PAB200_TC=1): groups of 9-32 query heads at D = 64, on
  // the 5th-generation tensor cores with TMEM accumulators; two warps per
  // ring, 64-token stages.
  pl->tc = pl->G > 8 && pl->G <= 32 && D == 64 && bs <= 64 && env_int("PAB200_TC", 0) != 0;
  if (pl->tc) pl->pair = true;
  if (pl->pair) pl->nt = 2;
  // Tokens per ring stage: a power of two >= block_size.
  pl->st = pl->tc ? 64 : env_int("PAB200_ST", bs <= 32 ? 32 : 64);
  if ((pl->st != 16 && pl->st != 32 && pl->st != 64) || pl->st < bs)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "PAB200_ST must be 16, 32 or 64 and >= block_size");
  const int nh = D / 64;
  if (2 * (pl->st / bs) * nh > 32)
    return fail(PAB200_ERR_UNSUPPORTED, "block_size %d with head_size %d needs > 32 copies per stage", bs, D);
  // Arithmetic: tensor-core MMA by default; the CUDA-core variant
  // (PAB200_CORE=1) exists for query groups of at most 4 heads, 32-token
  // stages and D <= 128.
  pl->core = env_int("PAB200_CORE", 0) != 0 && pl->G <= pab::kCoreMaxG && pl->st == 32 && D <= 128;
  if (pl->tc) pl->core = false;
  if (!select_kernel(a->dtype, D, pl->nt, pl->st, pl->core, pl->pair, pl->tc, &pl->ops))
    return fail(PAB200_ERR_UNSUPPORTED, "no kernel for head_size %d, group %d", D, pl->G);

  // Each warp owns a private ring of `depth` stages.  Throughput grows with
  // resident warps (each warp's stage loop is latency-bound), so the default
  // is a 2-deep ring and as many warps as ~200 KB of shared memory per SM
  // holds (6 warps at 16 KiB stages).
  const size_t stage = size_t(4) * pl->st * D;  // K + V bytes of one stage
  // The tcgen05 path computes the scores of the next stage while the warps
  // work on the current one, so it needs a third stage in flight.
  int depth = env_int("PAB200_DEPTH", pl->tc ? 3 : 2);
  if (depth < (pl->tc ? 3 : 2) || depth > pab::kMaxDepth)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "PAB200_DEPTH must be in [%d, %d]", pl->tc ? 3 : 2,
                pab::kMaxDepth);
  Geometry geo;
  if ((rc = choose_geometry(pl->ops, dev, depth, stage, pl->pair, pab::core_q_bytes(pl->core, D),
                            pl->tc, env_int("PAB200_WPC", 0), &geo)))
    return rc;
  const int wpc = geo.wpc, per_sm = geo.per_sm;
  pl->depth = depth;
  pl->wpc = wpc;
  pl->smem = geo.smem;
  pl->ctas_per_sm = per_sm;
  const int upc = pl->pair ? wpc / 2 : wpc;  // rings (work units) per CTA
  int W = sms * per_sm * upc;
  pl->n_heads = a->num_seqs * a->num_kv_heads;
  if (a->num_splits > 1) {
    const int64_t cap = int64_t(pl->n_heads) * a->num_splits;
    if (cap < W) W = static_cast<int>(cap);
  }
  pl->W = W;
  pl->grid = (W + upc - 1) / upc;
  // Partial-state slot: acc [G][D], m [G], l [G].
  pl->slot_floats = (pl->G * D + 2 * pl->G + 3) & ~3;
  // Workspace: a 256-byte header (status, weff, parity of the current call,
  // empty-head count, dynamic-tail header), then cum, wstart,
  // claim words, per-head segment ranges for two calls, the list of empty
  // heads and the partial slots (n_heads + W * (m_max + 1): one per (head,
  // segment) pair).  Under a scratch cap the tail chunk count per warp is
  // lowered until the workspace fits.
  int m_max = env_int("PAB200_STEAL_M", 4);
  if (m_max < 0) m_max = 0;
  for (;; --m_max) {
    size_t off = 256;
    pl->off_cum = off;
    off = align256(off + size_t(pl->n_heads + 1) * 4);
    pl->off_wstart = off;
    off = align256(off + size_t(W) * 4);
    pl->off_claims = off;
    off = align256(off + size_t(W) * 8);
    pl->off_hseg = off;
    off = align256(off + size_t(pl->n_heads) * 16);
    pl->off_empty = off;
    off = align256(off + size_t(pl->n_heads) * 4);
    pl->off_part = off;
    off = align256(off + (size_t(pl->n_heads) + size_t(W) * (m_max + 1)) * pl->slot_floats * 4);
    pl->ws_bytes = off;
    if (m_max == 0 || off <= scratch_cap) break;
  }
  pl->steal_m_max = m_max;
  pl->steal_min_stages = env_int("PAB200_STEAL_MIN_STAGES", 4);
  return PAB200_OK;
}

int encode_cache_map_uncached(const pab200_decode_args* a, const void* base, CUtensorMap* map);

// Tensor maps depend only on the cache pointer and its geometry; calls on the
// same caches reuse the last few encodings instead of re-encoding per call.
int encode_cache_map(const pab200_decode_args* a, const void* base, CUtensorMap* map) {
  struct Entry {
    const void* base;
    int64_t pages;
    int32_t dtype, layout, D, bs, hkv;
    CUtensorMap map;
  };
  constexpr int kEntries = 8;
  static Entry cache[kEntries];
  static int used = 0, next = 0;
  static std::mutex mu;
  const int32_t hkv = a->layout == PAB200_LAYOUT_NHD ? a->num_kv_heads : 1;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i) {
      const Entry& e = cache[i];
      if (e.base == base && e.pages == a->num_pages && e.dtype == a->dtype &&
          e.layout == a->layout && e.D == a->head_size && e.bs == a->block_size && e.hkv == hkv) {
        *map = e.map;
        return PAB200_OK;
      }
    }
  }
  int rc = encode_cache_map_uncached(a, base, map);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(mu);
  cache[next] = Entry{base, a->num_pages, a->dtype, a->layout, a->head_size, a->block_size, hkv, *map};
  next = (next + 1) % kEntries;
  if (used < kEntries) ++used;
  return PAB200_OK;
}

int encode_cache_map_uncached(const pab200_decode_args* a, const void* base, CUtensorMap* map) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(PAB200_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int D = a->head_size;
  const uint64_t hc = a->layout == PAB200_LAYOUT_NHD ? uint64_t(a->num_kv_heads) : 1u;
  cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(hc),
                        cuuint64_t(a->num_pages) * cuuint64_t(a->block_size)};
  cuuint64_t strides[2] = {cuuint64_t(D) * 2, cuuint64_t(hc) * D * 2};
  cuuint32_t box[3] = {64, 1, cuuint32_t(a->block_size)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map,
                   a->dtype == PAB200_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PAB200_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return PAB200_OK;
}

// The planner is launched with programmatic dependent launch: it may start
// while the previous call's kernels on this stream still run (the previous
// reduce kernel lets it start once every reduce CTA has read its parity),
// loads and plans, and writes the workspace only after they have finished.
template <typename T>
cudaError_t launch_plan(const pab::DecodeParams& p, cudaStream_t s, bool pdl) {
  LaunchCfg lc(dim3(1), dim3(1024), 0, s, pdl);
  if (p.append) return cudaLaunchKernelEx(&lc.cfg, pab::plan_kernel<T, true>, p);
  return cudaLaunchKernelEx(&lc.cfg, pab::plan_kernel<T, false>, p);
}


}  // namespace

namespace {
// Reduce launch: while heads hold few partial states, one warp per head (or
// per (head, query head) row when G * D > 1024); when they hold many, one CTA
// (4 warps splitting the partials) per row.  The expected count assumes every
// head as long as its block table allows: the warps' static ranges plus the
// tail chunks the planner would cut for that many pages (the planner's own
// choice, on the device, depends on the actual lengths).
double expected_spans(const Plan& pl, const pab::DecodeParams& p) {
  const int64_t pages = int64_t(pl.n_heads) * (p.maxb > 0 ? p.maxb : 1);
  const int W = static_cast<int>(pages < pl.W ? pages : pl.W);
  int m = 0, k = 0;
  pab::tail_chunks(pages, W, pl.steal_m_max, pl.st / p.bs, pl.steal_min_stages, &m, &k);
  return double(W) * (m + 1) / pl.n_heads + 1.0;
}

template <typename T, int D, int NCT>
cudaError_t launch_reduce_heads(const pab::DecodeParams& p, int n_heads, cudaStream_t s, bool pdl) {
  LaunchCfg lc(dim3(static_cast<unsigned>((n_heads + 3) / 4)), dim3(128), 0, s, pdl);
  return cudaLaunchKernelEx(&lc.cfg, pab::reduce_heads_kernel<T, D, NCT>, p);
}

template <typename T, int D>
cudaError_t launch_reduce_d(const pab::DecodeParams& p, const Plan& pl, cudaStream_t s, bool pdl) {
  int nct = 1;  // float4 output chunks per lane: G*D/128 rounded up to a power of two
  while (nct * 128 < pl.G * D) nct *= 2;
  // Dependent rounds of partial-state loads: the warp-per-head (or per-row)
  // kernel keeps 16/nct (16) partials in flight per warp; the CTA-per-row
  // kernel splits a row's partials over 4 warps, 16 in flight each, and
  // spends about one more round combining them.  Either is run in waves of
  // about 4 resident 4-warp CTAs per SM.  The fewer rounds win; ties go to
  // the warp-per-head kernel (fewer CTAs).
  const double spans = expected_spans(pl, p);
  const double in_flight = nct > 8 ? 16.0 : 16.0 / nct;
  const int64_t rows = int64_t(pl.n_heads) * pl.G;
  const double per_wave = 4.0 * device_sm_count_current();
  const double ctas_heads =
      std::ceil(double(nct > 8 ? rows : pl.n_heads) / (nct > 8 && D < 128 ? 4.0 * (128 / D) : 4.0));
  const double rounds_heads = std::ceil(spans / in_flight) * std::ceil(ctas_heads / per_wave);
  const double rounds_split = (std::ceil(spans / 64.0) + 1.0) * std::ceil(double(rows) / per_wave);
  if (rounds_heads <= rounds_split) {
    switch (nct) {
      case 1: return launch_reduce_heads<T, D, 1>(p, pl.n_heads, s, pdl);
      case 2: return launch_reduce_heads<T, D, 2>(p, pl.n_heads, s, pdl);
      case 4: return launch_reduce_heads<T, D, 4>(p, pl.n_heads, s, pdl);
      case 8: return launch_reduce_heads<T, D, 8>(p, pl.n_heads, s, pdl);
      default: {  // G*D > 1024: one warp (D = 64: half-warp) per (head, query head) row
        const int64_t per_cta = D < 128 ? 4 * (128 / D) : 4;
        LaunchCfg lc(dim3(static_cast<unsigned>((rows + per_cta - 1) / per_cta)), dim3(128), 0, s,
                     pdl);
        return cudaLaunchKernelEx(&lc.cfg, pab::reduce_rows_kernel<T, D>, p);
      }
    }
  }
  LaunchCfg lc(dim3(static_cast<unsigned>(rows)), dim3(128), 0, s, pdl);
  return cudaLaunchKernelEx(&lc.cfg, pab::reduce_split_kernel<T, D>, p);
}

template <typename T>
cudaError_t launch_reduce(const pab::DecodeParams& p, const Plan& pl, cudaStream_t s, bool pdl) {
  switch (p.D) {
    case 64: return launch_reduce_d<T, 64>(p, pl, s, pdl);
    case 128: return launch_reduce_d<T, 128>(p, pl, s, pdl);
    default: return launch_reduce_d<T, 256>(p, pl, s, pdl);
  }
}
}  // namespace

PAB200_EXPORT size_t pab200_decode_workspace_size(const pab200_decode_args* args) {
  Plan pl;
  if (make_plan(args, &pl, SIZE_MAX) != PAB200_OK) return 0;
  return pl.ws_bytes;
}

PAB200_EXPORT int pab200_decode_launch_count(const pab200_decode_args* args) {
  Plan pl;
  if (make_plan(args, &pl, SIZE_MAX) != PAB200_OK) return 0;
  return 3;
}

namespace {
cudaError_t launch_exchange(const pab::ExchangeParams& p, int out_dtype, int fused_d,
                            cudaStream_t s);

// One decode call planned as `pl`; with `app`, the planner first appends the
// step's tokens; with `exchange`, the call ends in the fused exchange + merge
// of a context split across GPUs instead of the reduce kernel.
int decode_impl(const pab200_decode_args* a, const Plan& pl, const pab::AppendParams* app,
                void* workspace, size_t workspace_bytes, void* stream,
                pab::ExchangeParams* exchange = nullptr, int exchange_dtype = 0) {
  int rc = PAB200_OK;
  if (!workspace || workspace_bytes < pl.ws_bytes)
    return fail(PAB200_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", pl.ws_bytes,
                workspace ? workspace_bytes : size_t(0));
  if (!aligned(workspace, 256)) return fail(PAB200_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);

  pab::DecodeParams p{};
  p.out = a->out;
  p.q = a->q;
  p.lens = a->seqlens;
  p.bt = a->block_table;
  p.q_sb = a->q_stride_b;
  p.q_sh = a->q_stride_h;
  p.o_sb = a->out_stride_b;
  p.o_sh = a->out_stride_h;
  p.l_sb = a->seqlens_stride_b;
  p.l_sh = a->seqlens_stride_h;
  p.bt_sb = a->bt_stride_b;
  p.bt_sh = a->bt_stride_h;
  p.bt_si = a->bt_stride_i;
  p.bt_mul = a->bt_page_mul;
  p.bt_add = a->bt_page_add;
  p.B = a->num_seqs;
  p.Hkv = a->num_kv_heads;
  p.G = pl.G;
  p.D = a->head_size;
  p.bs = a->block_size;
  p.maxb = a->max_blocks;
  p.num_pages = a->num_pages;
  p.head_in_map = a->layout == PAB200_LAYOUT_NHD ? 1 : 0;
  p.scale_log2 = a->softmax_scale * pab::kLog2e;
  p.total_warps = pl.W;
  p.depth = pl.depth;
  p.status = reinterpret_cast<uint32_t*>(ws);
  p.weff = reinterpret_cast<int32_t*>(ws + 4);
  p.steal = reinterpret_cast<int32_t*>(ws + 16);
  p.claims = reinterpret_cast<unsigned long long*>(ws + pl.off_claims);
  p.hseg = reinterpret_cast<int4*>(ws + pl.off_hseg);
  p.parity = reinterpret_cast<uint32_t*>(ws + 8);
  p.n_empty = reinterpret_cast<int32_t*>(ws + 12);
  p.empty = reinterpret_cast<int32_t*>(ws + pl.off_empty);
  p.steal_m_max = pl.steal_m_max;
  p.steal_pps = pl.st / a->block_size;
  p.steal_min_stages = pl.steal_min_stages;
  p.cum = reinterpret_cast<int32_t*>(ws + pl.off_cum);
  p.wstart = reinterpret_cast<int32_t*>(ws + pl.off_wstart);
  p.part = reinterpret_cast<float*>(ws + pl.off_part);
  p.slot_floats = pl.slot_floats;
  p.state_o = a->state_o;
  p.state_lse = a->state_lse;
  p.append = app ? 1 : 0;
  // Early start of the decode grid (see DecodeParams::early): not with an
  // append (the planner writes the lengths and the cache the decode reads)
  // nor with mma.sync warp pairs, and only while the prefix fits shared
  // memory (the tcgen05 path keeps it in its operand tiles).
  p.early = !app && (!pl.pair || pl.tc) && pl.n_heads <= pab::kEarlyMaxHeads &&
            env_int("PAB200_EARLY", 1) != 0;
  if (app) {
    p.app = *app;
    p.app.status = p.status;  // append bits land in the call's status word
  }

  CUtensorMap kmap, vmap;
  if (a->num_pages > 0) {
    if ((rc = encode_cache_map(a, a->k_cache, &kmap))) return rc;
    if ((rc = encode_cache_map(a, a->v_cache, &vmap))) return rc;
  } else {
    // No pages: every sequence is empty, the planner writes all outputs and
    // the decode kernel exits before touching the maps.
    kmap = CUtensorMap{};
    vmap = CUtensorMap{};
  }

  const bool pdl = env_int("PAB200_PDL", 1) != 0;
  cudaError_t e = a->dtype == PAB200_DTYPE_BF16 ? launch_plan<__nv_bfloat16>(p, s, pdl)
                                                 : launch_plan<__half>(p, s, pdl);
  if (e != cudaSuccess) return cuda_fail(e, "plan kernel launch");
  if (a->event_before) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a->event_before), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  e = pl.ops.launch(dim3(pl.grid), dim3(pl.wpc * 32), pl.smem, s, pdl && !a->event_before, kmap,
                    vmap, p);
  if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
  if (a->event_after) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a->event_after), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  if (exchange) {
    // Context split across GPUs: the exchange + merge kernel folds the split
    // heads' partial states itself (no reduce kernel).
    exchange->part = p.part;
    exchange->hseg = p.hseg;
    exchange->parity = p.parity;
    exchange->slot_floats = p.slot_floats;
    exchange->G = p.G;
    e = launch_exchange(*exchange, exchange_dtype, p.D, s);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "exchange kernel launch");
    return PAB200_OK;
  }
  const bool pdl_r = pdl && !a->event_after;
  e = a->dtype == PAB200_DTYPE_BF16 ? launch_reduce<__nv_bfloat16>(p, pl, s, pdl_r)
                                    : launch_reduce<__half>(p, pl, s, pdl_r);
  if (e != cudaSuccess) return cuda_fail(e, "reduce kernel launch");
  return PAB200_OK;
}
}  // namespace

PAB200_EXPORT int pab200_decode(const pab200_decode_args* a, void* workspace,
                                size_t workspace_bytes, void* stream) {
  Plan pl;
  const int rc = make_plan(a, &pl, SIZE_MAX);
  if (rc) return rc;
  return decode_impl(a, pl, nullptr, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------- no-alloc
// Fixed scratch for callers that cannot provide a workspace (see
// pab200_decode_noalloc in pab200.h).  In host code `g_noalloc_scratch` names
// a host-side stand-in, not device memory: its device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[PAB200_NOALLOC_SCRATCH_BYTES];

namespace {

int noalloc_scratch(void** out) {
  static void* ptrs[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(PAB200_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return PAB200_OK;
}

}  // namespace

PAB200_EXPORT int pab200_decode_noalloc(const pab200_decode_args* a, void* stream) {
  Plan pl;
  int rc = make_plan(a, &pl, PAB200_NOALLOC_SCRATCH_BYTES);
  if (rc) return rc;
  if (pl.ws_bytes > PAB200_NOALLOC_SCRATCH_BYTES)
    return fail(PAB200_ERR_WORKSPACE,
                "this call needs %zu bytes of scratch but the fixed no-alloc scratch holds %u; "
                "use pab200_decode with a caller workspace",
                pl.ws_bytes, PAB200_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  if ((rc = noalloc_scratch(&ws))) return rc;
  return decode_impl(a, pl, nullptr, ws, PAB200_NOALLOC_SCRATCH_BYTES, stream);
}

namespace {
// Arguments of the flat north-star entry point: the reference page layout,
// every tensor contiguous.
pab200_decode_args flat_args(void* out, const void* query, const void* key_cache,
                             const void* value_cache, const int32_t* block_tables,
                             const int32_t* context_lens, float scale, int32_t block_size,
                             int32_t dtype, int32_t num_seqs, int32_t num_q_heads,
                             int32_t num_kv_heads, int32_t head_size, int32_t max_blocks,
                             int64_t num_pages) {
  pab200_decode_args a{};
  a.out = out;
  a.q = query;
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.seqlens = context_lens;
  a.block_table = block_tables;
  a.dtype = dtype;
  a.layout = PAB200_LAYOUT_PAGES;
  a.num_seqs = num_seqs;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_size = head_size;
  a.block_size = block_size;
  a.max_blocks = max_blocks;
  a.num_pages = num_pages;
  a.q_stride_b = int64_t(num_q_heads) * head_size;
  a.q_stride_h = head_size;
  a.out_stride_b = int64_t(num_q_heads) * head_size;
  a.out_stride_h = head_size;
  a.seqlens_stride_b = num_kv_heads;
  a.seqlens_stride_h = 1;
  a.bt_stride_b = int64_t(num_kv_heads) * max_blocks;
  a.bt_stride_h = max_blocks;
  a.bt_stride_i = 1;
  a.bt_page_mul = 1;
  a.bt_page_add = 0;
  a.softmax_scale = scale;
  a.num_splits = 0;
  return a;
}
}  // namespace

PAB200_EXPORT size_t pab200_paged_attention_workspace_size(int32_t dtype, int32_t num_seqs,
                                                           int32_t num_q_heads,
                                                           int32_t num_kv_heads,
                                                           int32_t head_size,
                                                           int32_t block_size,
                                                           int32_t max_blocks,
                                                           int64_t num_pages) {
  const pab200_decode_args a =
      flat_args(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 1.f, block_size, dtype,
                num_seqs, num_q_heads, num_kv_heads, head_size, max_blocks, num_pages);
  Plan pl;
  if (make_plan(&a, &pl, SIZE_MAX, /*check_pointers=*/false) != PAB200_OK) return 0;
  return pl.ws_bytes;
}

PAB200_EXPORT int pab200_paged_attention(void* out, const void* query, const void* key_cache,
                                         const void* value_cache, const int32_t* block_tables,
                                         const int32_t* context_lens, float scale,
                                         int32_t block_size, int32_t dtype, int32_t num_seqs,
                                         int32_t num_q_heads, int32_t num_kv_heads,
                                         int32_t head_size, int32_t max_blocks, int64_t num_pages,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  const pab200_decode_args a =
      flat_args(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                block_size, dtype, num_seqs, num_q_heads, num_kv_heads, head_size, max_blocks,
                num_pages);
  return pab200_decode(&a, workspace, workspace_bytes, stream);
}

PAB200_EXPORT int pab200_merge_states(const float* state_o, int64_t o_stride,
                                      const float* state_lse, int64_t lse_stride,
                                      int32_t num_states, int64_t rows, int32_t head_size,
                                      void* out, int64_t out_stride_row, int32_t out_dtype,
                                      void* stream) {
  if (num_states < 1 || rows < 0 || head_size < 4 || (head_size & 3))
    return fail(PAB200_ERR_INVALID_ARGUMENT, "num_states >= 1, rows >= 0, head_size %% 4 == 0 required");
  if (rows == 0) return PAB200_OK;
  if (!state_o || !state_lse || !out) return fail(PAB200_ERR_INVALID_ARGUMENT, "null pointer");
  if (num_states > 1 && (o_stride < rows * head_size || lse_stride < rows))
    return fail(PAB200_ERR_INVALID_ARGUMENT, "state strides smaller than one state");
  const size_t oal = out_dtype == PAB200_DTYPE_F32 ? 16 : 8;
  if (!aligned(state_o, 16) || (o_stride & 3) || !aligned(out, oal) || (out_stride_row & 3))
    return fail(PAB200_ERR_ALIGNMENT,
                "state_o 16-byte aligned with o_stride %% 4 == 0, out %zu-byte aligned, "
                "out_stride_row %% 4 == 0", oal);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8)), block(256);
  switch (out_dtype) {
    case PAB200_DTYPE_BF16:
      pab::merge_states_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(
          state_o, o_stride, state_lse, lse_stride, num_states, rows, head_size,
          static_cast<__nv_bfloat16*>(out), out_stride_row);
      break;
    case PAB200_DTYPE_F16:
      pab::merge_states_kernel<__half><<<grid, block, 0, s>>>(
          state_o, o_stride, state_lse, lse_stride, num_states, rows, head_size,
          static_cast<__half*>(out), out_stride_row);
      break;
    case PAB200_DTYPE_F32:
      pab::merge_states_kernel<float><<<grid, block, 0, s>>>(
          state_o, o_stride, state_lse, lse_stride, num_states, rows, head_size,
          static_cast<float*>(out), out_stride_row);
      break;
    default:
      return fail(PAB200_ERR_UNSUPPORTED, "out_dtype %d", out_dtype);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
  return PAB200_OK;
}

namespace {
int64_t packed_state_floats(int64_t rows, int32_t head_size) {
  return rows * head_size + ((rows + 3) / 4) * 4;
}
int64_t exchange_epoch_words(int64_t rows) { return ((pab::exchange_blocks(rows) + 3) / 4) * 4; }
}  // namespace

PAB200_EXPORT size_t pab200_exchange_buffer_bytes(int32_t world, int64_t rows, int32_t head_size) {
  if (world < 1 || rows < 1 || head_size < 4 || (head_size & 3)) return 0;
  return size_t(2 * world * packed_state_floats(rows, head_size)) * 8 +
         size_t(exchange_epoch_words(rows)) * 4;
}

PAB200_EXPORT int pab200_exchange_buffer_create(size_t bytes, void** buf, void* ipc_handle) {
  if (!bytes || !buf || !ipc_handle) return fail(PAB200_ERR_INVALID_ARGUMENT, "null pointer or size 0");
  *buf = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (exchange buffer)");
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "exchange buffer setup");
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *buf = p;
  return PAB200_OK;
}

PAB200_EXPORT int pab200_exchange_buffer_open(const void* ipc_handle, void** peer_buf) {
  if (!ipc_handle || !peer_buf) return fail(PAB200_ERR_INVALID_ARGUMENT, "null pointer");
  *peer_buf = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return PAB200_OK;
}

PAB200_EXPORT int pab200_exchange_buffer_reset(void* buf, size_t bytes, void* stream) {
  if (!buf) return fail(PAB200_ERR_INVALID_ARGUMENT, "null pointer");
  cudaError_t e = cudaMemsetAsync(buf, 0, bytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PAB200_OK : cuda_fail(e, "cudaMemsetAsync");
}

PAB200_EXPORT int pab200_exchange_buffer_close(void* peer_buf) {
  if (!peer_buf) return PAB200_OK;
  cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
  return e == cudaSuccess ? PAB200_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

PAB200_EXPORT int pab200_exchange_buffer_destroy(void* buf) {
  if (!buf) return PAB200_OK;
  cudaError_t e = cudaFree(buf);
  return e == cudaSuccess ? PAB200_OK : cuda_fail(e, "cudaFree");
}

namespace {
// Checks the arguments of an exchange + merge and fills its parameters
// (without the fused-decode fields).
int exchange_params(float* state, void* const* bufs, int32_t rank, int32_t world, int64_t rows,
                    int32_t head_size, void* out, int64_t out_stride_row, int32_t out_dtype,
                    int64_t wait_limit_ns, uint32_t* status, pab::ExchangeParams* p) {
  if (world < 1 || world > 64 || rank < 0 || rank >= world || rows < 1 || head_size < 4 ||
      (head_size & 3) || wait_limit_ns <= 0)
    return fail(PAB200_ERR_INVALID_ARGUMENT,
                "need 0 <= rank < world <= 64, rows >= 1, head_size %% 4 == 0, wait_limit_ns > 0");
  if (!state || !bufs || !out || !status) return fail(PAB200_ERR_INVALID_ARGUMENT, "null pointer");
  if (out_dtype != PAB200_DTYPE_BF16 && out_dtype != PAB200_DTYPE_F16 && out_dtype != PAB200_DTYPE_F32)
    return fail(PAB200_ERR_UNSUPPORTED, "out_dtype %d", out_dtype);
  const size_t oal = out_dtype == PAB200_DTYPE_F32 ? 16 : 8;
  if (!aligned(state, 16) || !aligned(out, oal) || (out_stride_row & 3) || !aligned(status, 4))
    return fail(PAB200_ERR_ALIGNMENT, "state 16-byte, out %zu-byte aligned, out_stride_row %% 4 == 0",
                oal);
  *p = pab::ExchangeParams{};
  p->state = state;
  p->bufs = reinterpret_cast<uint64_t* const*>(bufs);
  p->rank = rank;
  p->world = world;
  p->S = packed_state_floats(rows, head_size);
  p->rows = rows;
  p->D = head_size;
  p->out = out;
  p->out_stride = out_stride_row;
  p->wait_limit_ns = static_cast<uint64_t>(wait_limit_ns);
  p->status = status;
  // Every rank uses the same grid: block b owns rows [b*rpb, (b+1)*rpb) on
  // all ranks and waits only for the peers' block b.
  const int64_t blocks = pab::exchange_blocks(rows);
  p->rows_per_block = (rows + blocks - 1) / blocks;
  return PAB200_OK;
}

// Programmatic dependent launch: the grid is scheduled while the kernel
// that writes `state` drains, and waits for it (griddepcontrol.wait) before
// the first read.  fused_d: 0, or the head size when the kernel first folds
// the split heads' partial states of the decode call before it.
template <typename TO>
cudaError_t launch_exchange_t(const pab::ExchangeParams& p, int fused_d, cudaStream_t s) {
  LaunchCfg lc(dim3(static_cast<unsigned>(pab::exchange_blocks(p.rows))), dim3(256), 0, s, true);
  switch (fused_d) {
    case 0: return cudaLaunchKernelEx(&lc.cfg, pab::exchange_merge_kernel<TO, 0>, p);
    case 64: return cudaLaunchKernelEx(&lc.cfg, pab::exchange_merge_kernel<TO, 64>, p);
    case 128: return cudaLaunchKernelEx(&lc.cfg, pab::exchange_merge_kernel<TO, 128>, p);
    default: return cudaLaunchKernelEx(&lc.cfg, pab::exchange_merge_kernel<TO, 256>, p);
  }
}

cudaError_t launch_exchange(const pab::ExchangeParams& p, int out_dtype, int fused_d,
                            cudaStream_t s) {
  switch (out_dtype) {
    case PAB200_DTYPE_BF16: return launch_exchange_t<__nv_bfloat16>(p, fused_d, s);
    case PAB200_DTYPE_F16: return launch_exchange_t<__half>(p, fused_d, s);
    default: return launch_exchange_t<float>(p, fused_d, s);
  }
}
}  // namespace

PAB200_EXPORT int pab200_exchange_merge(const float* state, void* const* bufs, int32_t rank,
                                        int32_t world, int64_t rows, int32_t head_size, void* out,
                                        int64_t out_stride_row, int32_t out_dtype,
                                        int64_t wait_limit_ns, uint32_t* status, void* stream) {
  pab::ExchangeParams p;
  const int rc = exchange_params(const_cast<float*>(state), bufs, rank, world, rows, head_size, out,
                                 out_stride_row, out_dtype, wait_limit_ns, status, &p);
  if (rc) return rc;
  cudaError_t e = launch_exchange(p, out_dtype, 0, static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "exchange kernel launch");
  return PAB200_OK;
}

PAB200_EXPORT int pab200_decode_exchange(const pab200_decode_args* a, void* workspace,
                                         size_t workspace_bytes, void* const* bufs, int32_t rank,
                                         int32_t world, void* out, int64_t out_stride_row,
                                         int32_t out_dtype, int64_t wait_limit_ns,
                                         uint32_t* status, void* stream) {
  if (!a) return fail(PAB200_ERR_INVALID_ARGUMENT, "args is null");
  const int64_t rows = int64_t(a->num_seqs) * a->num_q_heads;
  if (!a->state_o || !a->state_lse || a->state_lse != a->state_o + rows * a->head_size)
    return fail(PAB200_ERR_INVALID_ARGUMENT,
                "state_o / state_lse must be this rank's packed state (lse right after o)");
  pab::ExchangeParams ep;
  int rc = exchange_params(a->state_o, bufs, rank, world, rows, a->head_size, out, out_stride_row,
                           out_dtype, wait_limit_ns, status, &ep);
  if (rc) return rc;
  Plan pl;
  if ((rc = make_plan(a, &pl, SIZE_MAX))) return rc;
  return decode_impl(a, pl, nullptr, workspace, workspace_bytes, stream, &ep, out_dtype);
}

namespace {
// Validates a KV append and fills its kernel parameters.  Returns
// PAB200_OK, or an error (num_seqs == 0 sets *empty).
int append_params(const pab200_kv_append_args* a, pab::AppendParams* out, bool* empty) {
  *empty = false;
  if (!a) return fail(PAB200_ERR_INVALID_ARGUMENT, "args is null");
  if (a->dtype != PAB200_DTYPE_BF16 && a->dtype != PAB200_DTYPE_F16)
    return fail(PAB200_ERR_UNSUPPORTED, "dtype %d: caches must be bf16 or f16", a->dtype);
  if (a->layout != PAB200_LAYOUT_PAGES && a->layout != PAB200_LAYOUT_NHD)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "unknown cache layout %d", a->layout);
  if (a->num_seqs < 0 || a->num_kv_heads < 1 || a->block_size < 1 || a->max_blocks < 1 ||
      a->head_size < 2 || (a->head_size & 1) || a->head_size > 256 || a->num_pages < 0)
    return fail(PAB200_ERR_INVALID_ARGUMENT,
                "need num_seqs >= 0, num_kv_heads, block_size, max_blocks >= 1, even head_size <= 256");
  if (a->num_seqs == 0) {
    *empty = true;
    return PAB200_OK;
  }
  if (!a->k_cache || !a->v_cache || !a->k_new || !a->v_new || !a->seqlens || !a->block_table)
    return fail(PAB200_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned(a->k_cache, 4) || !aligned(a->v_cache, 4) || !aligned(a->k_new, 4) ||
      !aligned(a->v_new, 4) || (a->new_stride_b & 1) || (a->new_stride_h & 1))
    return fail(PAB200_ERR_ALIGNMENT, "caches and new rows 4-byte aligned, even strides");
  pab::AppendParams& p = *out;
  p = pab::AppendParams{};
  p.k_cache = static_cast<uint32_t*>(a->k_cache);
  p.v_cache = static_cast<uint32_t*>(a->v_cache);
  p.k_new = static_cast<const uint32_t*>(a->k_new);
  p.v_new = static_cast<const uint32_t*>(a->v_new);
  p.lens = a->seqlens;
  p.bt = a->block_table;
  p.status = a->status;
  p.B = a->num_seqs;
  p.Hkv = a->num_kv_heads;
  p.D = a->head_size;
  p.bs = a->block_size;
  p.maxb = a->max_blocks;
  p.head_in_page = a->layout == PAB200_LAYOUT_NHD ? 1 : 0;
  p.num_pages = a->num_pages;
  p.n_sb = a->new_stride_b;
  p.n_sh = a->new_stride_h;
  p.l_sb = a->seqlens_stride_b;
  p.l_sh = a->seqlens_stride_h;
  p.bt_sb = a->bt_stride_b;
  p.bt_sh = a->bt_stride_h;
  p.bt_si = a->bt_stride_i;
  p.bt_mul = a->bt_page_mul;
  p.bt_add = a->bt_page_add;
  p.increment = a->increment ? 1 : 0;
  // 16-byte row copies when every row start is 16-byte aligned
  p.vec16 = aligned(a->k_cache, 16) && aligned(a->v_cache, 16) && aligned(a->k_new, 16) &&
            aligned(a->v_new, 16) && (a->new_stride_b % 8 == 0) && (a->new_stride_h % 8 == 0) &&
            (a->head_size % 8 == 0);
  return PAB200_OK;
}
}  // namespace

PAB200_EXPORT int pab200_kv_append(const pab200_kv_append_args* a, void* stream) {
  pab::AppendParams p;
  bool empty = false;
  const int rc = append_params(a, &p, &empty);
  if (rc || empty) return rc;
  pab::kv_append_kernel<<<(a->num_seqs + 3) / 4, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PAB200_OK : cuda_fail(e, "kv append launch");
}

PAB200_EXPORT int pab200_decode_append(const pab200_decode_args* a, const pab200_kv_append_args* app,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!a || !app) return fail(PAB200_ERR_INVALID_ARGUMENT, "args is null");
  pab::AppendParams p;
  bool empty = false;
  int rc = append_params(app, &p, &empty);
  if (rc) return rc;
  // The append must address the cache, table and lengths this call decodes.
  if (app->k_cache != a->k_cache || app->v_cache != a->v_cache ||
      app->block_table != a->block_table || app->seqlens != a->seqlens ||
      app->dtype != a->dtype || app->layout != a->layout || app->num_seqs != a->num_seqs ||
      app->num_kv_heads != a->num_kv_heads || app->head_size != a->head_size ||
      app->block_size != a->block_size || app->max_blocks != a->max_blocks ||
      app->num_pages != a->num_pages || app->seqlens_stride_b != a->seqlens_stride_b ||
      app->seqlens_stride_h != a->seqlens_stride_h || app->bt_stride_b != a->bt_stride_b ||
      app->bt_stride_h != a->bt_stride_h || app->bt_stride_i != a->bt_stride_i ||
      app->bt_page_mul != a->bt_page_mul || app->bt_page_add != a->bt_page_add)
    return fail(PAB200_ERR_INVALID_ARGUMENT,
                "append arguments must name the decode call's caches, block table and lengths");
  Plan pl;
  if ((rc = make_plan(a, &pl, SIZE_MAX))) return rc;
  return decode_impl(a, pl, empty ? nullptr : &p, workspace, workspace_bytes, stream);
}

PAB200_EXPORT int pab200_read_status(const void* workspace, uint32_t* status_out, void* stream) {
  if (!workspace || !status_out) return fail(PAB200_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status_out, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the status word");
  return PAB200_OK;
}

PAB200_EXPORT const char* pab200_strerror(int status) {
  switch (status) {
    case PAB200_OK: return "ok";
    case PAB200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PAB200_ERR_UNSUPPORTED: return "unsupported configuration";
    case PAB200_ERR_WORKSPACE: return "workspace missing or too small";
    case PAB200_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case PAB200_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

PAB200_EXPORT const char* pab200_last_error(void) { return g_last_error; }

PAB200_EXPORT int pab200_abi_version(void) { return PAB200_ABI_VERSION; }

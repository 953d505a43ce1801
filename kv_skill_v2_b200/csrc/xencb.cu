// libxencb: the C ABI (include/xencb.h) over the sm_100a kernels of the Library read.
//
// Host side of every entry point: validate arguments (XENCB_EINVAL with a message, the reference's
// ValueError), plan the launch from the device's SM count, check the caller's workspace, launch on the
// caller's stream. No entry point allocates device memory or synchronises, except xencb_device_status.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cudaTypedefs.h>
#include <unordered_map>
#include <atomic>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "project.cuh"
#include "gemm_tc.cuh"
#include "gemm_f16x3.cuh"
#include "read_decode.cuh"
#include "read_decode_mma.cuh"
#include "read_multi.cuh"
#include "prefill.cuh"
#include "route.cuh"
#include "library_build.cuh"
#include "topk_read.cuh"
#include "attn.cuh"
#include "exchange.cuh"

// Scratch of xencb_read_decode_noalloc: a fixed device array, so that entry point never allocates.
static __device__ __align__(256) unsigned char g_noalloc_scratch[XENCB_NOALLOC_SCRATCH_BYTES];

namespace xencb {
namespace {

thread_local std::string g_err;
// events of xencb_read_kernel_events, consumed by the next read launch on this thread
thread_local cudaEvent_t g_read_ev_before = nullptr, g_read_ev_after = nullptr;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(XENCB_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// Kernels this library has launched (or captured into a graph) in this process; every launch site checks
// its launch through XENCB_CHECK_LAUNCH_N, which also counts it.
std::atomic<unsigned long long> g_launches{0};

#define XENCB_CHECK_LAUNCH_N(what, n)                    \
  do {                                                   \
    cudaError_t e__ = cudaGetLastError();                \
    if (e__ != cudaSuccess) return cuda_fail(e__, what); \
    g_launches.fetch_add((n), std::memory_order_relaxed); \
  } while (0)
#define XENCB_CHECK_LAUNCH(what) XENCB_CHECK_LAUNCH_N(what, 1)

// Launch with programmatic stream serialisation (the kernel may be scheduled while the one before it in the stream
// drains; it holds its dependent work behind pdl_wait(), common.cuh). Only kernels written for it go through
// here. XENCB_PDL=0 in the environment launches them plainly. A failed launch is reported by the
// XENCB_CHECK_LAUNCH that follows (the runtime records it for cudaGetLastError).
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("XENCB_PDL");
    return !(e && e[0] == '0' && e[1] == 0);
  }();
  return on;
}

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  (void)cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

constexpr int kMaxDev = 64;

struct DevInfo {
  int sms = 0;
  int max_smem_optin = 0;
};

DevInfo g_dev[kMaxDev];
std::mutex g_mu;

int device_info(DevInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return fail(XENCB_ENOTSUP, "device ordinal %d out of range", dev);
  if (g_dev[dev].sms == 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_dev[dev].sms == 0) {
      int sms = 0, smem = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
      e = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem opt-in)");
      g_dev[dev].max_smem_optin = smem;
      g_dev[dev].sms = sms;
    }
  }
  *out = g_dev[dev];
  return XENCB_OK;
}

int elem_size(int dtype) {
  switch (dtype) {
    case XENCB_F32: return 4;
    case XENCB_F16: return 2;
    case XENCB_BF16: return 2;
    default: return 0;
  }
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Opt a kernel into `smem` bytes of dynamic shared memory once per (device, kernel).
std::unordered_map<const void*, int> g_smem_set[kMaxDev];
std::mutex g_smem_mu;

template <typename K>
int ensure_smem(K kernel, int smem) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDev) return fail(XENCB_ENOTSUP, "device ordinal %d out of range", dev);
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lk(g_smem_mu);
  auto itr = g_smem_set[dev].find(key);
  if (itr != g_smem_set[dev].end() && itr->second >= smem) return XENCB_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  g_smem_set[dev][key] = smem;
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ GEMM plan
// Tensor-core path (gemm_tc.cuh) when the rows can be TMA-described (K % 4 == 0, 16-byte aligned bases);
// otherwise the SIMT fallback. The workspace covers either, so its size does not depend on pointer values.
struct GemmPlan {
  bool tc;
  int splits, kps;
  size_t part_bytes;
};

GemmPlan plan_gemm_tc(int64_t M, int N, int K, int sms) {
  GemmPlan p;
  p.tc = true;
  const int64_t tiles = ((N + TC_BM - 1) / TC_BM) * ((M + TC_BN - 1) / TC_BN);
  const int kblocks = (K + TC_BK - 1) / TC_BK;
  int64_t s = sms / tiles;  // one CTA per SM (the stage ring takes most of the shared memory)
  if (s < 1) s = 1;
  if (s > kblocks) s = kblocks;
  p.kps = (int)((kblocks + s - 1) / s) * TC_BK;
  p.splits = (K + p.kps - 1) / p.kps;
  p.part_bytes = align_up((size_t)p.splits * (size_t)M * (size_t)N * sizeof(float), 256);
  return p;
}

GemmPlan plan_gemm_simt(int64_t M, int N, int K, int sms) {
  GemmPlan p;
  p.tc = false;
  p.splits = sg_splits(M, N, K, sms);
  p.kps = sg_kps(K, p.splits);
  p.splits = (K + p.kps - 1) / p.kps;
  p.part_bytes = align_up((size_t)p.splits * (size_t)M * (size_t)N * sizeof(float), 256);
  return p;
}

// Workspace of a projection GEMM: the split partials of whichever kernel runs (the largest of the plans), then
// (tensor-core paths) the X staging: float32 X for the 3xTF32 kernel, or [X_hi; X_lo] f16 (the same bytes)
// plus one float per row for the 3xF16 kernels.
size_t gemm_part_bytes(int64_t M, int N, int K, int sms) {
  size_t b = plan_gemm_simt(M, N, K, sms).part_bytes;
  if (K % 4 == 0) b = std::max(b, plan_gemm_tc(M, N, K, (M > H3_BN ? 2 : 1) * sms).part_bytes);
  return b;
}

size_t gemm_xstage_bytes(int64_t M, int K) {
  return align_up((size_t)M * K * sizeof(float), 256) + align_up((size_t)M * sizeof(float), 256);
}

size_t gemm_ws_bytes(int64_t M, int N, int K, int sms, bool convert_x) {
  (void)convert_x;
  return gemm_part_bytes(M, N, K, sms) + (K % 4 == 0 ? gemm_xstage_bytes(M, K) : 0);
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B);

int tensor_map_f32_2d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                      uint32_t box_outer) {
  return tensor_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, inner, outer, inner * 4, box_inner, box_outer);
}

// A 2-D tensor map with 128- or 64-byte swizzle (the canonical UMMA operand layouts), OOB elements filled with
// zeros.
int tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swz) {
  if (!g_encode) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(XENCB_ECUDA, "cannot resolve cuTensorMapEncodeTiled from the driver");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  (void)esize;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box,
                              es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(XENCB_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return XENCB_OK;
}

// part = split partials of X @ W^T. X: [M, K] of type TX; W: [N, K] float32 (nn.Linear layout).
// `xbuf` (M*K float32, may be null when TX is float) stages a 16-bit X as float32 for the TMA path.
template <typename TX>
int launch_gemm(const void* X, int64_t M, int K, const float* W, int N, int sms, float* part, float* xbuf,
                int* row_done, cudaStream_t st, GemmPlan* used, const void* w_prep = nullptr) {
  // 3xF16 (weights split once by xencb_weights_prep, X split here with a power-of-two scale per row) whenever the
  // prepared weights are given: half the MMAs of 3xTF32, and no per-k-block split of W
  const bool f16x3 = w_prep != nullptr;
  if (f16x3 && K % 8 == 0 && aligned(w_prep, 256) && aligned(X, 16) && xbuf && M <= INT32_MAX / 2 &&
      N <= INT32_MAX / 2 && wprep_pairs(N, K) * 2 * H3_BM <= INT32_MAX) {
    const bool two = M > H3_BN;  // more than one row tile: two CTAs per SM (see gemm_f16x3.cuh)
    const GemmPlan p = plan_gemm_tc(M, N, K, (two ? 2 : 1) * sms);
    __half* xs = reinterpret_cast<__half*>(xbuf);  // [X_hi; X_lo]: 2 M K halves = M K floats of staging
    float* x_inv = reinterpret_cast<float*>(reinterpret_cast<char*>(xbuf) + align_up((size_t)M * K * sizeof(float), 256));
    launch_pdl(split_rows_f16x2_kernel<TX>, dim3((unsigned)M), dim3(SR_THREADS), 0, st, static_cast<const TX*>(X), M,
               K, xs, xs + M * (int64_t)K, x_inv);
    XENCB_CHECK_LAUNCH("split_rows_f16x2 launch");
    const char* wp = static_cast<const char*>(w_prep);
    CUtensorMap mw, mx;
    // the prepared tiles as one [pairs * 256, 64] f16 matrix: a box of 256 rows is one tile pair (W_hi, W_lo)
    int rc = tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, wp + WPREP_HEAD, H3_BK,
                           (uint64_t)wprep_pairs(N, K) * 2 * H3_BM, H3_BK * 2, H3_BK, 2 * H3_BM);
    if (rc) return rc;
    rc = tensor_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xs, (uint64_t)K, 2 * (uint64_t)M, (uint64_t)K * 2,
                       H3_BK, H3_BN);
    if (rc) return rc;
    auto kern = two ? gemm_f16x3_kernel<2, 2> : gemm_f16x3_kernel<4, 1>;
    const size_t h3s = h3_smem(two ? 2 : 4);
    rc = ensure_smem(kern, (int)h3s);
    if (rc) return rc;
    dim3 grid((N + H3_BM - 1) / H3_BM, (unsigned)((M + H3_BN - 1) / H3_BN), p.splits);
    launch_pdl(kern, grid, dim3(H3_THREADS), h3s, st, mw, mx, M, N, K, p.kps,
               reinterpret_cast<const float*>(wp) + 1, x_inv, part, row_done);
    XENCB_CHECK_LAUNCH("gemm_f16x3 launch");
    *used = p;
    return XENCB_OK;
  }
  const bool tc_ok = (K % 4 == 0) && aligned(W, 16) && (std::is_same<TX, float>::value ? aligned(X, 16) : xbuf != nullptr);
  if (tc_ok) {
    const GemmPlan p = plan_gemm_tc(M, N, K, sms);
    const float* xf = static_cast<const float*>(X);
    if (!std::is_same<TX, float>::value) {
      const int64_t n = M * (int64_t)K;
      to_f32_kernel<TX><<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, st>>>(static_cast<const TX*>(X),
                                                                                            n, xbuf);
      XENCB_CHECK_LAUNCH("to_f32 launch");
      xf = xbuf;
    }
    CUtensorMap mw, mx;
    int rc = tensor_map_f32_2d(&mw, W, (uint64_t)K, (uint64_t)N, TC_BOX, TC_BM);
    if (rc) return rc;
    rc = tensor_map_f32_2d(&mx, xf, (uint64_t)K, (uint64_t)M, TC_BOX, TC_BN);
    if (rc) return rc;
    rc = ensure_smem(gemm_tc_kernel, (int)TC_SMEM);
    if (rc) return rc;
    dim3 grid((N + TC_BM - 1) / TC_BM, (unsigned)((M + TC_BN - 1) / TC_BN), p.splits);
    gemm_tc_kernel<<<grid, TC_THREADS, TC_SMEM, st>>>(mw, mx, M, N, K, p.kps, part, row_done);
    XENCB_CHECK_LAUNCH("gemm_tc launch");
    *used = p;
    return XENCB_OK;
  }
  const GemmPlan p = plan_gemm_simt(M, N, K, sms);
  dim3 grid((N + SG_BN - 1) / SG_BN, (unsigned)((M + SG_BM - 1) / SG_BM), p.splits);
  gemm_simt_splitk_kernel<TX><<<grid, SG_THREADS, 0, st>>>(static_cast<const TX*>(X), M, K, W, N, p.kps, part,
                                                           row_done);
  XENCB_CHECK_LAUNCH("gemm_simt launch");
  *used = p;
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ read plan
struct ReadPlan {
  bool mma;  // tensor-core kernel (f16 / bf16 slots, d_s % 16 == 0, d_s <= 2560)
  int tpw;   // its 16-column tiles per consumer warp (8 or 16)
  int vpt, ncw, rps, n_stage, n_split, split_rows, row_bytes, row_stride, nvec, threads, grid;
  size_t smem, acc_bytes, ml_bytes;
  int64_t n_items;
  bool sparse;        // items listed by read_compact_kernel (xencb_read_decode_sparse)
  size_t list_bytes;  // its item list and count, after the partials
};

int plan_read(int64_t n_rows, int k, int d_s, int page_rows, int dtype, ReadPlan* p, bool untied = false,
              bool sparse = false) {
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int es = elem_size(dtype);
  if (!es) return fail(XENCB_EINVAL, "slots_dtype %d is not one of XENCB_F32/F16/BF16", dtype);
  if (d_s <= 0 || (int64_t)d_s * es % 16 != 0)
    return fail(XENCB_EINVAL, "d_s=%d: a slot row must be a multiple of 16 bytes (d_s %% %d == 0)", d_s, 16 / es);
  p->row_bytes = d_s * es;
  p->nvec = p->row_bytes / 16;
  const size_t budget = (size_t)(di.max_smem_optin > 0 ? di.max_smem_optin : 232448) - 1024;
  p->mma = false;
  const char* force_simt = getenv("XENCB_READ_SIMT");
  // tensor-core read: 128-column slices (up to 16 warps) for d_s <= 2048, 256-column slices (up to 10) above;
  // XENCB_READ_TPW=8|16 overrides the slice width (tuning)
  int tpw = d_s <= 2048 ? 8 : 16;
  if (const char* e = getenv("XENCB_READ_TPW")) {
    if (e[0] == '8' && e[1] == 0) tpw = 8;
    if (e[0] == '1' && e[1] == '6' && e[2] == 0) tpw = 16;
  }
  const int mma_ncw = (d_s + 16 * tpw - 1) / (16 * tpw);
  const int max_ncw = tpw == 8 ? RM_MAX_WARPS : 10;
  if ((dtype == XENCB_F16 || dtype == XENCB_BF16) && d_s % 16 == 0 && mma_ncw <= max_ncw &&
      !(force_simt && force_simt[0] == '1')) {
    const int stride = p->row_bytes + 16;
    int rps = 64;
    while (rps > 16 && rps * stride > 69632) rps >>= 1;
    if (untied) rps = 16;  // a key stage holds one 16-row group; its value stage follows
    const int stage_bytes = (int)align_up((size_t)rps * stride, 128);
    int n_stage = 8;
    while (n_stage >= 2 && rm_smem_bytes(n_stage, stage_bytes, mma_ncw, tpw) > budget) --n_stage;
    if (n_stage >= 2) {
      p->mma = true;
      p->tpw = tpw;
      p->vpt = 0;
      p->ncw = mma_ncw;
      p->threads = 32 * (mma_ncw + 2);  // producer + consumers + softmax warp
      p->rps = rps;
      p->row_stride = stride;
      p->n_stage = n_stage;
      p->smem = rm_smem_bytes(n_stage, stage_bytes, mma_ncw, tpw);
    }
  }
  if (!p->mma && untied)
    return fail(XENCB_ENOTSUP, "untied values are read by the tensor-core kernel only (f16 / bf16 slots, d_s %% 16 == 0)");
  if (!p->mma) {
    // at most 15 consumer warps (512 threads per CTA with the producer warp)
    if (p->nvec <= 15 * 32) p->vpt = 1;
    else if (p->nvec <= 15 * 64) p->vpt = 2;
    else return fail(XENCB_ENOTSUP, "d_s=%d: slot rows above 15 KiB are not supported", d_s);
    p->ncw = (p->nvec + 32 * p->vpt - 1) / (32 * p->vpt);
    p->threads = 32 * (p->ncw + 1);
    // rows per stage: a power of two <= 64 with a stage of about 32 KiB
    int rps = 64;
    while (rps > 1 && rps * p->row_bytes > 32768) rps >>= 1;
    p->rps = rps;
    p->row_stride = p->row_bytes;
    const size_t stage_bytes = align_up((size_t)rps * p->row_bytes, 128);
    const size_t tail = align_up(2 * (size_t)p->ncw * RD_G * sizeof(float), 8) + 2 * 8 * 8 + 16;
    int n_stage = (int)((budget - tail) / stage_bytes);
    if (n_stage > 8) n_stage = 8;
    if (n_stage < 2) return fail(XENCB_ENOTSUP, "d_s=%d: two pipeline stages do not fit in shared memory", d_s);
    p->n_stage = n_stage;
    p->smem = (size_t)n_stage * stage_bytes + align_up(2 * (size_t)p->ncw * RD_G * sizeof(float), 8) +
              2 * (size_t)n_stage * 8 + 16;
  }
  // row splits: pick the count with the smallest modelled makespan on one CTA per SM
  const int64_t pairs = n_rows * k;
  const int grid_max = di.sms;
  // (at most MERGE_ENTRIES splits: the merge keeps one chunk's coefficients in one batch)
  const int max_split = std::min(page_rows > 64 ? (page_rows + 63) / 64 : 1, MERGE_ENTRIES);
  double best = 1e300;
  int best_n = 1, best_rows = page_rows;
  for (int n = 1; n <= max_split; ++n) {
    int rows = page_rows;
    if (n > 1) rows = ((page_rows + n - 1) / n + 63) / 64 * 64;
    const int n_eff = (page_rows + rows - 1) / rows;
    if (n_eff != n) continue;
    const int64_t items = pairs * n_eff;
    const int64_t rounds = (items + grid_max - 1) / grid_max;
    const double cost = (double)rounds * ((double)rows * p->row_bytes + 8.0 * d_s * 4 + 16384.0);
    if (cost < best * 0.999) { best = cost; best_n = n_eff; best_rows = rows; }
  }
  p->n_split = best_n;
  p->split_rows = best_rows < 1 ? 1 : best_rows;
  p->sparse = false;
  p->list_bytes = 0;
  const int sp_split = std::min((page_rows + 127) / 128, MERGE_ENTRIES);
  if (sparse && p->mma && !untied && pairs <= 65536 && pairs * sp_split <= INT32_MAX) {  // one CTA lists them
    // sparse plan: 128-row pieces (eight 16-row stages; the merge then takes one batch of 16 entries per row at
    // top-4), only the pieces that hold rows listed on the device, so that a read where few rows take part
    // still spreads over every SM
    p->sparse = true;
    p->n_split = sp_split;
    p->split_rows = (page_rows + sp_split - 1) / sp_split;
    p->split_rows = (p->split_rows + 15) / 16 * 16;
    p->list_bytes = align_up((size_t)pairs * sp_split * sizeof(int32_t), 256) + 256;
  }
  p->n_items = pairs * p->n_split;
  p->grid = (int)(p->n_items < grid_max ? p->n_items : grid_max);
  if (p->grid < 1) p->grid = 1;
  p->acc_bytes = align_up((size_t)p->n_items * d_s * sizeof(float), 256);
  p->ml_bytes = align_up((size_t)p->n_items * 2 * sizeof(float), 256);
  return XENCB_OK;
}

template <typename TD>
void launch_sel_apply(const void* delta, const void* h, int h_dtype, int64_t n_rows, int d, const float* w,
                             int n_cand, int pos, float alpha, void* out, cudaStream_t st) {
  const TD* dp = static_cast<const TD*>(delta);
  TD* op = static_cast<TD*>(out);
  switch (h_dtype) {
    case XENCB_F32:
      selector_apply_kernel<TD, float><<<(unsigned)n_rows, 256, 0, st>>>(dp, static_cast<const float*>(h), d, w,
                                                                         n_cand, pos, alpha, op);
      break;
    case XENCB_F16:
      selector_apply_kernel<TD, __half><<<(unsigned)n_rows, 256, 0, st>>>(dp, static_cast<const __half*>(h), d, w,
                                                                          n_cand, pos, alpha, op);
      break;
    default:
      selector_apply_kernel<TD, __nv_bfloat16><<<(unsigned)n_rows, 256, 0, st>>>(
          dp, static_cast<const __nv_bfloat16*>(h), d, w, n_cand, pos, alpha, op);
      break;
  }
}

// Device address of g_noalloc_scratch on the current device, looked up once per device. Host code cannot use
// the array's name as a device pointer (it names a host-side shadow), so the address comes from the runtime.
void* g_noalloc_ptr[kMaxDev];
std::mutex g_noalloc_mu;

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return fail(XENCB_ENOTSUP, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    if (p == nullptr) return fail(XENCB_ECUDA, "cudaGetSymbolAddress returned a null scratch address");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return XENCB_OK;
}

struct MultiPlan {
  int tpw, ncw, threads, rps, row_bytes, row_stride, n_stage, grid, pieces, piece_rows, s_max, q_blocks;
  bool split;
  int64_t n_groups, units_per_group, n_units;
  size_t smem, fold_bytes, finfo_bytes, open_bytes, oinfo_bytes, mpart_bytes, mcount_bytes, soff_bytes, scoef_bytes,
      scount_bytes;
  int n_slabs;
  size_t total() const {
    return fold_bytes + finfo_bytes + open_bytes + oinfo_bytes + mpart_bytes + mcount_bytes + soff_bytes + scoef_bytes +
           scount_bytes;
  }
};

int plan_multi(int64_t n_rows, int64_t rows_per_lib, int n_chunks, int d_s, int page_rows, int dtype, MultiPlan* p,
               bool untied = false) {
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (dtype != XENCB_F16 && dtype != XENCB_BF16)
    return fail(XENCB_ENOTSUP, "read_multi: slots must be f16 or bf16 (f32 slots: use read_decode)");
  if (d_s <= 0 || d_s % 16 != 0) return fail(XENCB_ENOTSUP, "read_multi: d_s=%d must be a multiple of 16", d_s);
  p->tpw = d_s <= 2048 ? 8 : 16;
  p->ncw = (d_s + 16 * p->tpw - 1) / (16 * p->tpw);
  if (p->ncw > (p->tpw == 8 ? RM_MAX_WARPS : 10))
    return fail(XENCB_ENOTSUP, "read_multi: d_s=%d above 2560 is not supported", d_s);
  p->split = dtype == XENCB_BF16;
  p->threads = 32 * (p->ncw + 1);
  p->row_bytes = d_s * 2;
  p->row_stride = p->row_bytes + 16;
  int rps = 16;
  while (!untied && rps < 64 && 2 * rps * p->row_stride <= 36864) rps *= 2;  // untied: one group per key stage
  p->rps = rps;
  const int stage_bytes = (int)align_up((size_t)rps * p->row_stride, 128);
  const size_t budget = (size_t)(di.max_smem_optin > 0 ? di.max_smem_optin : 232448) - 1024;
  int n_stage = 8;
  while (n_stage >= 2 && mq_smem_bytes(n_stage, stage_bytes, p->ncw, p->tpw, p->split) > budget) --n_stage;
  if (n_stage < 2) return fail(XENCB_ENOTSUP, "read_multi: d_s=%d: two stages do not fit in shared memory", d_s);
  p->n_stage = n_stage;
  p->smem = mq_smem_bytes(n_stage, stage_bytes, p->ncw, p->tpw, p->split);
  const int64_t libs_used = (n_rows + rows_per_lib - 1) / rows_per_lib;
  const int64_t t_eff = rows_per_lib < n_rows ? rows_per_lib : n_rows;
  p->q_blocks = (int)((t_eff + MQ - 1) / MQ);
  p->n_groups = libs_used * p->q_blocks;
  // pieces: cut chunks until every CTA has at least 32 units (load balance within 1/32), pieces >= 32 rows
  int pieces = 1, piece_rows = page_rows;
  while (p->n_groups * n_chunks * pieces < 32LL * di.sms && piece_rows > 32) {
    pieces *= 2;
    piece_rows = (int)align_up((size_t)((page_rows + pieces - 1) / pieces), 16);
    if (piece_rows < 32) piece_rows = 32;
    pieces = (page_rows + piece_rows - 1) / piece_rows;
  }
  p->pieces = pieces;
  p->piece_rows = piece_rows;
  p->units_per_group = (int64_t)n_chunks * pieces;
  p->n_units = p->n_groups * p->units_per_group;
  p->grid = (int)(p->n_units < di.sms ? p->n_units : di.sms);
  if (p->grid < 1) p->grid = 1;
  if (p->grid > MM_MERGE_MAX_CTAS) return fail(XENCB_ENOTSUP, "read_multi: %d SMs exceed the merge's slot table", di.sms);
  const int64_t lmax = (p->n_units + p->grid - 1) / p->grid;
  p->s_max = (int)((lmax - 1 + p->units_per_group - 1) / p->units_per_group + 1);
  p->fold_bytes = align_up((size_t)p->grid * p->s_max * MQ * d_s * sizeof(float), 256);
  p->finfo_bytes = align_up((size_t)p->grid * p->s_max * sizeof(int64_t), 256);
  p->open_bytes = align_up((size_t)p->grid * 2 * (MQ_OPEN + (size_t)MQ * d_s) * sizeof(float), 256);
  p->oinfo_bytes = align_up((size_t)p->grid * 2 * sizeof(int64_t), 256);
  p->n_slabs = (d_s + 127) / 128;
  p->mpart_bytes = align_up((size_t)p->n_groups * p->n_slabs * MM_SQ * MQ * 128 * sizeof(float), 256);
  p->mcount_bytes = align_up((size_t)p->n_groups * p->n_slabs * sizeof(int), 256);
  p->soff_bytes = align_up((size_t)p->n_groups * MM_SRC_PER_CTA * p->grid * sizeof(int64_t), 256);
  p->scoef_bytes = align_up((size_t)p->n_groups * MM_SRC_PER_CTA * p->grid * MQ * sizeof(float), 256);
  p->scount_bytes = align_up((size_t)p->n_groups * sizeof(int), 256);
  return XENCB_OK;
}


// Routing logits: a warp per (row, chunk) dot for decode; shared-memory tiles when a Library has many rows.
using rc_t = int;
rc_t launch_route_logits(const float* q, int64_t n_rows, int d_s, const float* S, int C, const int32_t* n_chunks_of,
                         int64_t rows_per_lib, float temp, float* logit, cudaStream_t st) {
  if (rows_per_lib >= 64) {
    const int64_t libs = (n_rows + rows_per_lib - 1) / rows_per_lib;
    dim3 grid((unsigned)((rows_per_lib + RT_ROWS - 1) / RT_ROWS), (unsigned)((C + RT_CH - 1) / RT_CH), (unsigned)libs);
    route_logits_tiled_kernel<<<grid, 256, 0, st>>>(q, n_rows, d_s, S, C, n_chunks_of, rows_per_lib, temp, logit);
    XENCB_CHECK_LAUNCH("route_logits_tiled launch");
    return XENCB_OK;
  }
  if (n_rows > INT32_MAX || (C + RL_CH - 1) / RL_CH > 65535)
    return fail(XENCB_EINVAL, "route: %lld rows x %d chunks exceed the launch grid", (long long)n_rows, C);
  const dim3 grid((unsigned)n_rows, (unsigned)((C + RL_CH - 1) / RL_CH));
  const size_t qsmem = (size_t)d_s * sizeof(float);
  if (qsmem <= 96 * 1024) {
    int rc = ensure_smem(route_logits_kernel<true>, (int)std::max<size_t>(qsmem, 48 * 1024));
    if (rc) return rc;
    route_logits_kernel<true><<<grid, 256, qsmem, st>>>(q, n_rows, d_s, S, C, n_chunks_of, rows_per_lib, temp, logit);
  } else {
    route_logits_kernel<false><<<grid, 256, 0, st>>>(q, n_rows, d_s, S, C, n_chunks_of, rows_per_lib, temp, logit);
  }
  XENCB_CHECK_LAUNCH("route_logits launch");
  return XENCB_OK;
}

}  // namespace
}  // namespace xencb

using namespace xencb;

// The wait self-test: one thread waits, with the given limit, on an mbarrier phase that nothing completes.
__global__ void wait_selftest_kernel(long long limit_cycles, int* result) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const bool ok = mbar_wait_spin_limit(&bar, 0, limit_cycles);
  if (result) *result = ok ? 1 : 0;
}

// Library build plan: splits per chunk and the column-sum workspace.
namespace {
struct BuildPlan {
  int n_split, split_rows, threads;
  size_t part_bytes;
};

int plan_build(int n_chunks, int d_s, int page_rows, BuildPlan* p) {
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (d_s > LB_MAX_THREADS * LB_VEC)
    return fail(XENCB_ENOTSUP, "library_build: d_s=%d above %d is not supported", d_s, LB_MAX_THREADS * LB_VEC);
  // splits: about eight CTAs per SM over all chunks (short waves, small tail), each split >= 4 row batches
  int want = (8 * di.sms + n_chunks - 1) / n_chunks;
  const int max_split = (page_rows + 4 * LB_ROWS - 1) / (4 * LB_ROWS);
  if (want > max_split) want = max_split;
  if (want < 1) want = 1;
  p->split_rows = (int)align_up((size_t)((page_rows + want - 1) / want), LB_ROWS);
  p->n_split = (page_rows + p->split_rows - 1) / p->split_rows;
  p->part_bytes = align_up((size_t)n_chunks * p->n_split * d_s * sizeof(float), 256);
  p->threads = (int)align_up((size_t)((d_s + LB_VEC - 1) / LB_VEC), 32);
  return XENCB_OK;
}
}  // namespace

extern "C" {

int xencb_abi_version(void) { return XENCB_ABI_VERSION; }

const char* xencb_last_error(void) { return g_err.c_str(); }

unsigned long long xencb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int xencb_device_status(void* stream, int clear, unsigned int* status_out) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_dev_status, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(status)");
  if (clear && v) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_dev_status, &z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(status)");
  }
  if (status_out) *status_out = v;
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ project_in
size_t xencb_project_in_workspace(int64_t n_rows, int d_m, int d_s) {
  DevInfo di;
  if (device_info(&di)) return 0;
  if (n_rows <= 0 || d_m <= 0 || d_s <= 0) return 0;
  const int nch = (d_s + PIN_CHUNK - 1) / PIN_CHUNK;
  return gemm_ws_bytes(n_rows, d_s, d_m, di.sms, true) + align_up((size_t)n_rows * nch * sizeof(float), 256) +
         align_up((size_t)n_rows * sizeof(int), 256);
}

// project_in, and (rf given) the fused decode routing of its rows: returns XENCB_ENOTSUP, launching nothing, when
// the fused form does not take the shape.
static int project_in_impl(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* w_in, const void* w_prep,
                           const float* b_in, int d_s, int flags, const float* gate_w, float gate_b,
                           const float* gate_b_dev, const float* sel_w, const float* sel_b, int n_cand, float rms_eps,
                           float* q_out, float* gate_out, float* rstd_out, float* z_out, void* workspace,
                           size_t workspace_bytes, void* stream, const RouteFuse* rf) {
  if (flags & ~(XENCB_PIN_RMS | XENCB_PIN_L2)) return fail(XENCB_EINVAL, "project_in: unknown flags 0x%x", flags);
  if (!h || (!w_in && !w_prep) || !q_out) return fail(XENCB_EINVAL, "project_in: h, w_in (or w_prep) and q_out are required");
  if (!w_in && (d_m % 8 != 0 || !aligned(w_prep, 256)))
    return fail(XENCB_EINVAL, "project_in: without w_in, w_prep must be 256-byte aligned and d_m %% 8 == 0");
  if (n_rows <= 0 || d_m <= 0 || d_s <= 0)
    return fail(XENCB_EINVAL, "project_in: n_rows=%lld d_m=%d d_s=%d must be positive", (long long)n_rows, d_m, d_s);
  if (!elem_size(h_dtype)) return fail(XENCB_EINVAL, "project_in: h_dtype %d unknown", h_dtype);
  if (gate_w && !gate_out) return fail(XENCB_EINVAL, "project_in: gate_w given without gate_out");
  if (d_s % 4 != 0 || !aligned(q_out, 16))
    return fail(XENCB_EINVAL, "project_in: d_s=%d must be a multiple of 4 and q_out 16-byte aligned", d_s);
  if (sel_w && (!z_out || n_cand <= 0 || n_cand > 32))
    return fail(XENCB_EINVAL, "project_in: selector needs z_out and 1 <= n_cand <= 32 (got %d)", n_cand);
  const size_t rf_smem = rf ? ((size_t)d_s + 2 * (size_t)rf->C) * sizeof(float) : 0;
  if (rf && (d_s > 12 * ROW_THREADS || !(flags & XENCB_PIN_L2) || rf->rows_per_lib >= 64 || rf_smem > 96 * 1024))
    return fail(XENCB_ENOTSUP, "project_in_route: the fused form takes decode rows (rows_per_lib < 64), L2-normalised "
                "q, d_s <= %d and d_s + 2 * C <= 24576 floats", 12 * ROW_THREADS);
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int nch = (d_s + PIN_CHUNK - 1) / PIN_CHUNK;
  const size_t g_bytes = gemm_ws_bytes(n_rows, d_s, d_m, di.sms, true);
  const size_t nq_bytes = align_up((size_t)n_rows * nch * sizeof(float), 256);
  const size_t need = g_bytes + nq_bytes + align_up((size_t)n_rows * sizeof(int), 256);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(XENCB_EINVAL, "project_in: workspace needs %zu bytes, 256-byte aligned (got %zu)", need,
                workspace_bytes);
  char* ws = static_cast<char*>(workspace);
  float* part = reinterpret_cast<float*>(ws);
  float* nq_part = reinterpret_cast<float*>(ws + g_bytes);
  int* row_done = reinterpret_cast<int*>(ws + g_bytes + nq_bytes);
  // X staging for the tensor-core paths sits after the tensor-core partials
  float* xbuf = (d_m % 4 == 0) ? reinterpret_cast<float*>(ws + gemm_part_bytes(n_rows, d_s, d_m, di.sms)) : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmPlan gp;
  switch (h_dtype) {
    case XENCB_F32:
      rc = launch_gemm<float>(h, n_rows, d_m, w_in, d_s, di.sms, part, w_prep ? xbuf : nullptr, row_done, st, &gp,
                              w_prep);
      break;
    case XENCB_F16:
      rc = launch_gemm<__half>(h, n_rows, d_m, w_in, d_s, di.sms, part, xbuf, row_done, st, &gp, w_prep);
      break;
    default:
      rc = launch_gemm<__nv_bfloat16>(h, n_rows, d_m, w_in, d_s, di.sms, part, xbuf, row_done, st, &gp, w_prep);
      break;
  }
  if (rc) return rc;
  if (d_s <= 12 * ROW_THREADS) {  // one CTA per row: the reduce, 1/rms, bias and L2 norm in registers
    const int vpt = (d_s + 4 * ROW_THREADS - 1) / (4 * ROW_THREADS);  // float4 columns per thread: 1..3
    const unsigned thr = (unsigned)std::min<int>(ROW_THREADS, (d_s / 4 + 31) / 32 * 32);
    const PinArgs pa{d_m, part, gp.splits, n_rows, d_s, flags, b_in, gate_w, gate_b, gate_b_dev, sel_w, sel_b,
                     n_cand, rms_eps, q_out, gate_out, rstd_out, z_out};
    int lrc = XENCB_OK;
    auto launch = [&](auto kern, const auto* hp) {
      launch_pdl(kern, dim3((unsigned)n_rows), dim3(thr), 0, st, hp, pa);
    };
    // Routing CTAs per row: enough to fill the SMs once (a row's summary keys through up to 8 SMs), when the call
    // has a [n_rows, C] output to pass the logits through. XENCB_ROUTE_CTAS=<n> in the environment fixes it.
    int G = 1;
    if (rf && (rf->logit_out || rf->w_dense)) {
      // dense shard routing reads every chunk: up to 32 CTAs per row there
      G = (int)std::max<int64_t>(1, std::min<int64_t>(rf->lse_header ? 32 : 8, di.sms / n_rows));
      if (const char* e = getenv("XENCB_ROUTE_CTAS")) G = std::max(1, std::min(8, atoi(e)));
      G = std::min(G, rf->C);
    }
    auto launch_rf = [&](auto kern, const auto* hp) {
      lrc = ensure_smem(kern, (int)std::max<size_t>(rf_smem, 48 * 1024));
      RouteFuse r2 = *rf;
      r2.xlg = rf->logit_out ? rf->logit_out : rf->w_dense;
      r2.done = row_done;
      if (!lrc) launch_pdl(kern, dim3((unsigned)n_rows, (unsigned)G), dim3(thr), rf_smem, st, hp, pa, r2);
    };
    auto by_vpt = [&](const auto* hp) {
      using TH = std::remove_const_t<std::remove_pointer_t<decltype(hp)>>;
      if (rf) {
        if (vpt == 1) launch_rf(project_in_route_kernel<TH, 1>, hp);
        else if (vpt == 2) launch_rf(project_in_route_kernel<TH, 2>, hp);
        else launch_rf(project_in_route_kernel<TH, 3>, hp);
      } else if (vpt == 1) {
        launch(project_in_row_kernel<TH, 1>, hp);
      } else if (vpt == 2) {
        launch(project_in_row_kernel<TH, 2>, hp);
      } else {
        launch(project_in_row_kernel<TH, 3>, hp);
      }
    };
    switch (h_dtype) {
      case XENCB_F32: by_vpt(static_cast<const float*>(h)); break;
      case XENCB_F16: by_vpt(static_cast<const __half*>(h)); break;
      default: by_vpt(static_cast<const __nv_bfloat16*>(h)); break;
    }
    if (lrc) return lrc;
    XENCB_CHECK_LAUNCH("project_in row launch");
    return XENCB_OK;
  }
#define XENCB_PIN(T)                                                                                         \
  project_in_reduce_kernel<T><<<dim3((unsigned)n_rows, nch), 256, 0, st>>>(                                   \
      static_cast<const T*>(h), d_m, part, gp.splits, n_rows, d_s, flags, b_in, gate_w, gate_b, gate_b_dev,      \
      sel_w, sel_b,                                                                                            \
      n_cand, rms_eps, q_out, nq_part, row_done, gate_out, rstd_out, z_out)
  switch (h_dtype) {
    case XENCB_F32: XENCB_PIN(float); break;
    case XENCB_F16: XENCB_PIN(__half); break;
    default: XENCB_PIN(__nv_bfloat16); break;
  }
#undef XENCB_PIN
  XENCB_CHECK_LAUNCH("project_in reduce launch");
  return XENCB_OK;
}

int xencb_project_in(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* w_in, const void* w_prep,
                     const float* b_in, int d_s, int flags, const float* gate_w, float gate_b, const float* gate_b_dev,
                     const float* sel_w, const float* sel_b, int n_cand, float rms_eps, float* q_out, float* gate_out,
                     float* rstd_out, float* z_out, void* workspace, size_t workspace_bytes, void* stream) {
  return project_in_impl(h, h_dtype, n_rows, d_m, w_in, w_prep, b_in, d_s, flags, gate_w, gate_b, gate_b_dev, sel_w,
                         sel_b, n_cand, rms_eps, q_out, gate_out, rstd_out, z_out, workspace, workspace_bytes, stream,
                         nullptr);
}

int xencb_project_in_route(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* w_in, const void* w_prep,
                           const float* b_in, int d_s, int flags, const float* gate_w, float gate_b,
                           const float* gate_b_dev, const float* sel_w, const float* sel_b, int n_cand, float rms_eps,
                           float* q_out, float* gate_out, float* rstd_out, float* z_out, const float* S, int n_chunks,
                           const int32_t* n_chunks_of, int64_t rows_per_lib, int64_t n_lib, float route_temp, int top_k,
                           const float* row_w, int32_t* idx, float* wk, float* w_dense, float* logit_out,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (!S || !idx || !wk) return fail(XENCB_EINVAL, "project_in_route: S, idx and wk are required");
  if (n_rows <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0)
    return fail(XENCB_EINVAL, "project_in_route: sizes must be positive (n_rows=%lld C=%d rows_per_lib=%lld "
                "n_lib=%lld)", (long long)n_rows, n_chunks, (long long)rows_per_lib, (long long)n_lib);
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "project_in_route: %lld rows at %lld rows per Library need more than %lld Libraries",
                (long long)n_rows, (long long)rows_per_lib, (long long)n_lib);
  if (top_k < 0) return fail(XENCB_EINVAL, "project_in_route: top_k=%d must be >= 0", top_k);
  if (!aligned(S, 16)) return fail(XENCB_EINVAL, "project_in_route: S must be 16-byte aligned");
  const RouteFuse rf{S,  n_chunks, n_chunks_of, rows_per_lib, route_temp, top_k, xencb_route_k(top_k, n_chunks),
                     row_w, idx, wk, w_dense, logit_out, nullptr, nullptr, nullptr};
  return project_in_impl(h, h_dtype, n_rows, d_m, w_in, w_prep, b_in, d_s, flags, gate_w, gate_b, gate_b_dev, sel_w,
                         sel_b, n_cand, rms_eps, q_out, gate_out, rstd_out, z_out, workspace, workspace_bytes, stream,
                         &rf);
}

int xencb_project_in_route_lse(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* w_in,
                               const void* w_prep, const float* b_in, int d_s, int flags, const float* gate_w,
                               float gate_b, const float* gate_b_dev, float rms_eps, float* q_out, float* gate_out,
                               float* rstd_out, const float* S, int n_chunks, const int32_t* n_chunks_of,
                               int64_t rows_per_lib, int64_t n_lib, float route_temp, float* w_out, float* header_out,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (!S || !w_out || !header_out) return fail(XENCB_EINVAL, "project_in_route_lse: S, w_out and header_out are required");
  if (n_rows <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0)
    return fail(XENCB_EINVAL, "project_in_route_lse: sizes must be positive");
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "project_in_route_lse: %lld rows at %lld rows per Library need more than %lld "
                "Libraries", (long long)n_rows, (long long)rows_per_lib, (long long)n_lib);
  if (!aligned(S, 16)) return fail(XENCB_EINVAL, "project_in_route_lse: S must be 16-byte aligned");
  const RouteFuse rf{S, n_chunks, n_chunks_of, rows_per_lib, route_temp, 0, 0, nullptr, nullptr, nullptr, w_out,
                     nullptr, nullptr, nullptr, header_out};
  return project_in_impl(h, h_dtype, n_rows, d_m, w_in, w_prep, b_in, d_s, flags, gate_w, gate_b, gate_b_dev,
                         nullptr, nullptr, 0, rms_eps, q_out, gate_out, rstd_out, nullptr, workspace, workspace_bytes,
                         stream, &rf);
}

int xencb_rms_norm(const void* h, int h_dtype, int64_t n_rows, int d_m, float eps, float* out, void* stream) {
  if (!h || !out) return fail(XENCB_EINVAL, "rms_norm: h and out are required");
  if (n_rows <= 0 || d_m <= 0) return fail(XENCB_EINVAL, "rms_norm: sizes must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (h_dtype) {
    case XENCB_F32: rms_norm_kernel<float><<<(unsigned)n_rows, 256, 0, st>>>(static_cast<const float*>(h), d_m, eps, out); break;
    case XENCB_F16: rms_norm_kernel<__half><<<(unsigned)n_rows, 256, 0, st>>>(static_cast<const __half*>(h), d_m, eps, out); break;
    case XENCB_BF16:
      rms_norm_kernel<__nv_bfloat16><<<(unsigned)n_rows, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(h), d_m, eps, out);
      break;
    default: return fail(XENCB_EINVAL, "rms_norm: h_dtype %d unknown", h_dtype);
  }
  XENCB_CHECK_LAUNCH("rms_norm launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ route
int xencb_route_k(int top_k, int n_chunks) { return (top_k > 0 && top_k < n_chunks) ? top_k : n_chunks; }

int xencb_route(const float* q, int64_t n_rows, int d_s, const float* S, int n_chunks, const int32_t* n_chunks_of,
                int64_t rows_per_lib, int64_t n_lib, float route_temp, int top_k, const float* row_w, int32_t* idx,
                float* wk, float* w_dense, float* logit_out, void* stream) {
  if (!q || !S || !idx || !wk) return fail(XENCB_EINVAL, "route: q, S, idx and wk are required");
  if (n_rows <= 0 || d_s <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0)
    return fail(XENCB_EINVAL, "route: sizes must be positive (n_rows=%lld d_s=%d C=%d rows_per_lib=%lld n_lib=%lld)",
                (long long)n_rows, d_s, n_chunks, (long long)rows_per_lib, (long long)n_lib);
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "route: %lld rows at %lld rows per Library need more than %lld Libraries",
                (long long)n_rows, (long long)rows_per_lib, (long long)n_lib);
  if (top_k < 0) return fail(XENCB_EINVAL, "route: top_k=%d must be >= 0", top_k);
  if ((size_t)n_chunks * 4 * TOPK_WARPS > 200 * 1024)
    return fail(XENCB_ENOTSUP, "route: C=%d chunks exceed the router's shared-memory row buffer", n_chunks);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int k_out = xencb_route_k(top_k, n_chunks);
  // decode (few rows per Library, up to 128 chunks: at most two dot products per warp): one launch, a cluster of
  // 64 warps per row (per 64 / C rows when C < 64)
  const int rpc = std::max(1, std::min(8, 64 / n_chunks));
  const size_t fsmem = (size_t)rpc * (d_s + 2 * (size_t)n_chunks) * sizeof(float);
  const int64_t n_clusters = (n_rows + rpc - 1) / rpc;
  if (rows_per_lib < 64 && n_chunks <= 128 && fsmem <= 96 * 1024 && n_clusters * RF_CL <= INT32_MAX) {
    int rc = ensure_smem(route_fused_kernel, (int)std::max<size_t>(fsmem, 48 * 1024));
    if (rc) return rc;
    // programmatic serialisation: the kernel requests its S rows before it waits for q (the input projection)
    launch_pdl(route_fused_kernel, dim3((unsigned)(n_clusters * RF_CL)), dim3(256), fsmem, st, q, n_rows, d_s, S,
               n_chunks, n_chunks_of, rows_per_lib, route_temp, rpc, top_k, k_out, row_w, idx, wk, w_dense,
               logit_out);
    XENCB_CHECK_LAUNCH("route_fused launch");
    return XENCB_OK;
  }
  // logits go to logit_out when given, else to w_dense, which the top-k pass then overwrites row by row
  float* lg = logit_out ? logit_out : w_dense;
  if (!lg) return fail(XENCB_EINVAL, "route: one of w_dense / logit_out must be given (logit buffer)");
  rc_t rl = launch_route_logits(q, n_rows, d_s, S, n_chunks, n_chunks_of, rows_per_lib, route_temp, lg, st);
  if (rl) return rl;
  const int smem = n_chunks * 4 * TOPK_WARPS;
  int rc = ensure_smem(route_topk_kernel, smem > 48 * 1024 ? smem : 48 * 1024);
  if (rc) return rc;
  route_topk_kernel<<<(unsigned)((n_rows + TOPK_WARPS - 1) / TOPK_WARPS), TOPK_WARPS * 32, smem, st>>>(
      lg, n_rows, n_chunks, n_chunks_of, rows_per_lib, top_k, k_out, row_w, idx, wk, w_dense);
  XENCB_CHECK_LAUNCH("route_topk launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ read
size_t xencb_read_decode_workspace(int64_t n_rows, int k, int d_s, int page_rows, int slots_dtype) {
  if (n_rows <= 0 || k <= 0 || d_s <= 0 || page_rows <= 0) return 0;
  ReadPlan p;
  if (plan_read(n_rows, k, d_s, page_rows, slots_dtype, &p)) return 0;
  return p.acc_bytes + p.ml_bytes;
}

size_t xencb_read_decode_sparse_workspace(int64_t n_rows, int k, int d_s, int page_rows, int slots_dtype) {
  if (n_rows <= 0 || k <= 0 || d_s <= 0 || page_rows <= 0) return 0;
  ReadPlan p;
  if (plan_read(n_rows, k, d_s, page_rows, slots_dtype, &p, false, true)) return 0;
  return p.acc_bytes + p.ml_bytes + p.list_bytes;
}

static int read_decode_impl(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                     int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of, const int32_t* n_valid,
                     int n_chunks, int64_t rows_per_lib, int64_t n_lib, const int32_t* idx, const float* wk, int k,
                     float read_temp, int read_softmax, float* r_out, void* workspace, size_t workspace_bytes,
                     void* stream, bool sparse) {
  if (!q || !slots || !page_of || !n_valid || !idx || !wk || !r_out)
    return fail(XENCB_EINVAL, "read_decode: q, slots, page_of, n_valid, idx, wk and r_out are required");
  if (n_rows <= 0 || d_s <= 0 || page_rows <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0 || k <= 0)
    return fail(XENCB_EINVAL, "read_decode: sizes must be positive");
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "read_decode: %lld rows need more than %lld Libraries", (long long)n_rows,
                (long long)n_lib);
  const int es = elem_size(slots_dtype);
  if (!es) return fail(XENCB_EINVAL, "read_decode: slots_dtype %d unknown", slots_dtype);
  if (n_pages <= 0) return fail(XENCB_EINVAL, "read_decode: n_pages=%lld must be positive", (long long)n_pages);
  if (page_stride < (int64_t)page_rows * d_s)
    return fail(XENCB_EINVAL, "read_decode: page_stride %lld < page_rows*d_s %lld", (long long)page_stride,
                (long long)page_rows * d_s);
  if (!aligned(slots, 16) || (page_stride * es) % 16 != 0 || !aligned(q, 16) || !aligned(r_out, 16))
    return fail(XENCB_EINVAL, "read_decode: slots, q, r_out and page_stride*elem must be 16-byte aligned");
  if (vslots && !aligned(vslots, 16)) return fail(XENCB_EINVAL, "read_decode: vslots must be 16-byte aligned");
  ReadPlan p;
  int rc = plan_read(n_rows, k, d_s, page_rows, slots_dtype, &p, vslots != nullptr, sparse);
  if (rc) return rc;
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < p.acc_bytes + p.ml_bytes + p.list_bytes)
    return fail(XENCB_EINVAL, "read_decode: workspace needs %zu bytes, 256-byte aligned (got %zu)",
                p.acc_bytes + p.ml_bytes + p.list_bytes, workspace_bytes);
  ReadArgs a;
  a.q = q; a.n_rows = n_rows; a.d_s = d_s;
  a.slots = static_cast<const char*>(slots);
  a.vslots = static_cast<const char*>(vslots);
  a.n_pages = n_pages;
  a.page_stride_bytes = page_stride * es;
  a.page_rows = page_rows;
  a.page_of = page_of; a.n_valid = n_valid; a.n_chunks = n_chunks; a.rows_per_lib = rows_per_lib;
  a.idx = idx; a.wk = wk; a.k = k;
  a.qscale = read_softmax ? read_temp * 1.4426950408889634f : 1.f;
  a.n_split = p.n_split; a.split_rows = p.split_rows; a.rps = p.rps; a.n_stage = p.n_stage;
  a.row_bytes = p.row_bytes; a.nvec = p.nvec; a.n_items = p.n_items; a.row_stride = p.row_stride;
  a.part_acc = static_cast<float*>(workspace);
  a.part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + p.acc_bytes);
  a.item_list = nullptr;
  a.n_active = nullptr;
  a.plan_pairs = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the sparse plan inside the tensor-core kernel when the pairs' prefix sums fit next to its shared memory
  // (XENCB_READ_PLAN_KERNEL=1 in the environment keeps the separate compaction kernel)
  const char* plan_env = getenv("XENCB_READ_PLAN_KERNEL");
  const size_t plan_bytes = align_up((size_t)(n_rows * k + 1) * sizeof(int), 16);
  DevInfo di2;
  const bool plan_inline = p.sparse && p.mma && n_rows * k <= RM_PLAN_PAIRS && !(plan_env && plan_env[0] == '1') &&
                           device_info(&di2) == XENCB_OK &&
                           p.smem + plan_bytes <= (size_t)(di2.max_smem_optin > 0 ? di2.max_smem_optin : 232448) - 1024;
  if (plan_inline) {
    a.plan_pairs = (int)(n_rows * k);
    p.smem += plan_bytes;
  } else if (p.sparse) {
    char* lb = static_cast<char*>(workspace) + p.acc_bytes + p.ml_bytes;
    int32_t* list = reinterpret_cast<int32_t*>(lb);
    int* n_act = reinterpret_cast<int*>(lb + p.list_bytes - 256);
    read_compact_kernel<<<1, RC_THREADS, 0, st>>>(a, list, n_act);
    XENCB_CHECK_LAUNCH("read_compact_kernel launch");
    a.item_list = list;
    a.n_active = n_act;
  }
  rc = XENCB_OK;
  {
    auto run = [&](auto tag_t, auto tag_v, auto tag_s) -> int {
      using T = typename decltype(tag_t)::type;
      constexpr int V = decltype(tag_v)::value;
      constexpr bool S = decltype(tag_s)::value;
      auto k1 = read_decode_kernel<T, V, S>;
      int r2 = ensure_smem(k1, (int)p.smem);
      if (r2) return r2;
      cudaEvent_t ev0 = g_read_ev_before, ev1 = g_read_ev_after;
      g_read_ev_before = g_read_ev_after = nullptr;
      if (ev0) cudaEventRecord(ev0, st);
      k1<<<p.grid, p.threads, p.smem, st>>>(a);
      XENCB_CHECK_LAUNCH("read_decode_kernel launch");
      if (ev1) cudaEventRecord(ev1, st);
      dim3 mg((unsigned)n_rows, (d_s + 511) / 512);
      launch_pdl(read_merge_kernel<S>, mg, dim3(MERGE_THREADS), 0, st, a, r_out);
      XENCB_CHECK_LAUNCH("read_merge_kernel launch");
      return XENCB_OK;
    };
    struct F32T { using type = float; };
    struct F16T { using type = __half; };
    struct BF16T { using type = __nv_bfloat16; };
    using V1 = std::integral_constant<int, 1>;
    using V2 = std::integral_constant<int, 2>;
    using ST = std::true_type;
    using SF = std::false_type;
    auto run_mma = [&](auto tag_t, auto tag_s, auto tag_w) -> int {
      using T = typename decltype(tag_t)::type;
      constexpr bool S = decltype(tag_s)::value;
      constexpr int W = decltype(tag_w)::value;
      constexpr bool SPLIT = std::is_same<T, __nv_bfloat16>::value;
      auto k1 = read_decode_mma_kernel<T, SPLIT, S, W>;
      int r2 = ensure_smem(k1, (int)p.smem);
      if (r2) return r2;
      cudaEvent_t ev0 = g_read_ev_before, ev1 = g_read_ev_after;
      g_read_ev_before = g_read_ev_after = nullptr;
      if (ev0) cudaEventRecord(ev0, st);
      launch_pdl(k1, dim3(p.grid), dim3(p.threads), p.smem, st, a);
      XENCB_CHECK_LAUNCH("read_decode_mma_kernel launch");
      if (ev1) cudaEventRecord(ev1, st);
      dim3 mg((unsigned)n_rows, (d_s + 511) / 512);
      launch_pdl(read_merge_kernel<S>, mg, dim3(MERGE_THREADS), 0, st, a, r_out);
      XENCB_CHECK_LAUNCH("read_merge_kernel launch");
      return XENCB_OK;
    };
    using W8 = std::integral_constant<int, 8>;
    using W16 = std::integral_constant<int, 16>;
    if (p.mma && p.tpw == 8) {
      if (slots_dtype == XENCB_F16) rc = read_softmax ? run_mma(F16T{}, ST{}, W8{}) : run_mma(F16T{}, SF{}, W8{});
      else rc = read_softmax ? run_mma(BF16T{}, ST{}, W8{}) : run_mma(BF16T{}, SF{}, W8{});
    } else if (p.mma) {
      if (slots_dtype == XENCB_F16) rc = read_softmax ? run_mma(F16T{}, ST{}, W16{}) : run_mma(F16T{}, SF{}, W16{});
      else rc = read_softmax ? run_mma(BF16T{}, ST{}, W16{}) : run_mma(BF16T{}, SF{}, W16{});
    } else if (slots_dtype == XENCB_F16) {
      if (p.vpt == 1) rc = read_softmax ? run(F16T{}, V1{}, ST{}) : run(F16T{}, V1{}, SF{});
      else rc = read_softmax ? run(F16T{}, V2{}, ST{}) : run(F16T{}, V2{}, SF{});
    } else if (slots_dtype == XENCB_BF16) {
      if (p.vpt == 1) rc = read_softmax ? run(BF16T{}, V1{}, ST{}) : run(BF16T{}, V1{}, SF{});
      else rc = read_softmax ? run(BF16T{}, V2{}, ST{}) : run(BF16T{}, V2{}, SF{});
    } else {
      if (p.vpt == 1) rc = read_softmax ? run(F32T{}, V1{}, ST{}) : run(F32T{}, V1{}, SF{});
      else rc = read_softmax ? run(F32T{}, V2{}, ST{}) : run(F32T{}, V2{}, SF{});
    }
  }
  return rc;
}

int xencb_read_decode(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                      int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of, const int32_t* n_valid,
                      int n_chunks, int64_t rows_per_lib, int64_t n_lib, const int32_t* idx, const float* wk, int k,
                      float read_temp, int read_softmax, float* r_out, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return read_decode_impl(q, n_rows, d_s, slots, vslots, slots_dtype, n_pages, page_stride, page_rows, page_of,
                          n_valid, n_chunks, rows_per_lib, n_lib, idx, wk, k, read_temp, read_softmax, r_out,
                          workspace, workspace_bytes, stream, false);
}

int xencb_read_decode_sparse(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots,
                             int slots_dtype, int64_t n_pages, int64_t page_stride, int page_rows,
                             const int32_t* page_of, const int32_t* n_valid, int n_chunks, int64_t rows_per_lib,
                             int64_t n_lib, const int32_t* idx, const float* wk, int k, float read_temp,
                             int read_softmax, float* r_out, void* workspace, size_t workspace_bytes, void* stream) {
  return read_decode_impl(q, n_rows, d_s, slots, vslots, slots_dtype, n_pages, page_stride, page_rows, page_of,
                          n_valid, n_chunks, rows_per_lib, n_lib, idx, wk, k, read_temp, read_softmax, r_out,
                          workspace, workspace_bytes, stream, true);
}

// ------------------------------------------------------------------------------------------------ read_multi
size_t xencb_read_multi_workspace(int64_t n_rows, int64_t rows_per_lib, int n_chunks, int d_s, int page_rows,
                                  int slots_dtype) {
  if (n_rows <= 0 || rows_per_lib <= 0 || n_chunks <= 0 || d_s <= 0 || page_rows <= 0) return 0;
  MultiPlan p;
  if (plan_multi(n_rows, rows_per_lib, n_chunks, d_s, page_rows, slots_dtype, &p)) return 0;
  return p.total();
}

int xencb_read_multi(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                     int64_t n_pages,
                     int64_t page_stride, int page_rows, const int32_t* page_of, const int32_t* n_valid, int n_chunks,
                     const int32_t* n_chunks_of, int64_t rows_per_lib, int64_t n_lib, const float* w, float read_temp,
                     int read_softmax, float* r_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !slots || !page_of || !n_valid || !w || !r_out)
    return fail(XENCB_EINVAL, "read_multi: q, slots, page_of, n_valid, w and r_out are required");
  if (n_rows <= 0 || d_s <= 0 || page_rows <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0)
    return fail(XENCB_EINVAL, "read_multi: sizes must be positive");
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "read_multi: %lld rows need more than %lld Libraries", (long long)n_rows,
                (long long)n_lib);
  if (n_pages <= 0) return fail(XENCB_EINVAL, "read_multi: n_pages=%lld must be positive", (long long)n_pages);
  if (page_stride < (int64_t)page_rows * d_s)
    return fail(XENCB_EINVAL, "read_multi: page_stride %lld < page_rows*d_s %lld", (long long)page_stride,
                (long long)page_rows * d_s);
  if (!aligned(slots, 16) || (page_stride * 2) % 16 != 0 || !aligned(q, 16) || !aligned(r_out, 16))
    return fail(XENCB_EINVAL, "read_multi: slots, q, r_out and page_stride*elem must be 16-byte aligned");
  if (vslots && !aligned(vslots, 16)) return fail(XENCB_EINVAL, "read_multi: vslots must be 16-byte aligned");
  MultiPlan p;
  int rc = plan_multi(n_rows, rows_per_lib, n_chunks, d_s, page_rows, slots_dtype, &p, vslots != nullptr);
  if (rc) return rc;
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < p.total())
    return fail(XENCB_EINVAL, "read_multi: workspace needs %zu bytes, 256-byte aligned (got %zu)", p.total(),
                workspace_bytes);
  MultiArgs a;
  a.q = q; a.n_rows = n_rows; a.d_s = d_s;
  a.slots = static_cast<const char*>(slots);
  a.vslots = static_cast<const char*>(vslots);
  a.n_pages = n_pages; a.page_stride_bytes = page_stride * 2; a.page_rows = page_rows;
  a.page_of = page_of; a.n_valid = n_valid; a.n_chunks = n_chunks; a.n_chunks_of = n_chunks_of;
  a.rows_per_lib = rows_per_lib; a.w = w;
  a.qscale = read_softmax ? read_temp * 1.4426950408889634f : 1.f;
  a.q_blocks = p.q_blocks; a.n_groups = p.n_groups; a.pieces = p.pieces; a.piece_rows = p.piece_rows;
  a.units_per_group = p.units_per_group; a.n_units = p.n_units; a.s_max = p.s_max;
  a.rps = p.rps; a.n_stage = p.n_stage; a.row_bytes = p.row_bytes; a.row_stride = p.row_stride;
  char* ws = static_cast<char*>(workspace);
  a.fold = reinterpret_cast<float*>(ws);
  a.fold_info = reinterpret_cast<int64_t*>(ws + p.fold_bytes);
  a.open = reinterpret_cast<float*>(ws + p.fold_bytes + p.finfo_bytes);
  a.open_info = reinterpret_cast<int64_t*>(ws + p.fold_bytes + p.finfo_bytes + p.open_bytes);
  MultiMergeArgs mm;
  mm.part = reinterpret_cast<float*>(ws + p.fold_bytes + p.finfo_bytes + p.open_bytes + p.oinfo_bytes);
  mm.counter = reinterpret_cast<int*>(ws + p.fold_bytes + p.finfo_bytes + p.open_bytes + p.oinfo_bytes + p.mpart_bytes);
  mm.n_slabs = p.n_slabs;
  {
    char* m2 = ws + p.fold_bytes + p.finfo_bytes + p.open_bytes + p.oinfo_bytes + p.mpart_bytes + p.mcount_bytes;
    mm.src_off = reinterpret_cast<int64_t*>(m2);
    mm.src_coef = reinterpret_cast<float*>(m2 + p.soff_bytes);
    mm.src_count = reinterpret_cast<int*>(m2 + p.soff_bytes + p.scoef_bytes);
  }
  a.merge_counter = mm.counter;
  a.n_merge_counters = p.n_groups * (int64_t)p.n_slabs;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto run = [&](auto tag_t, auto tag_s, auto tag_w) -> int {
    using T = typename decltype(tag_t)::type;
    constexpr bool S = decltype(tag_s)::value;
    constexpr int W = decltype(tag_w)::value;
    constexpr bool SPLIT = std::is_same<T, __nv_bfloat16>::value;
    auto k1 = read_multi_mma_kernel<T, SPLIT, S, W>;
    int r2 = ensure_smem(k1, (int)p.smem);
    if (r2) return r2;
    launch_pdl(k1, dim3(p.grid), dim3(p.threads), p.smem, st, a);
    XENCB_CHECK_LAUNCH("read_multi_mma_kernel launch");
    launch_pdl(read_multi_coef_kernel<S>, dim3((unsigned)p.n_groups), dim3(MM_MERGE_THREADS), 0, st, a, (int)p.grid,
               mm);
    XENCB_CHECK_LAUNCH("read_multi_coef_kernel launch");
    dim3 mg((unsigned)p.n_groups, (unsigned)p.n_slabs, MM_SQ);
    launch_pdl(read_multi_sum_kernel, mg, dim3(MM_MERGE_THREADS), 0, st, a, (int)p.grid, mm, r_out);
    XENCB_CHECK_LAUNCH("read_multi_sum_kernel launch");
    return XENCB_OK;
  };
  struct F16T { using type = __half; };
  struct BF16T { using type = __nv_bfloat16; };
  using ST = std::true_type;
  using SF = std::false_type;
  using W8 = std::integral_constant<int, 8>;
  using W16 = std::integral_constant<int, 16>;
  if (p.tpw == 8) {
    if (slots_dtype == XENCB_F16) rc = read_softmax ? run(F16T{}, ST{}, W8{}) : run(F16T{}, SF{}, W8{});
    else rc = read_softmax ? run(BF16T{}, ST{}, W8{}) : run(BF16T{}, SF{}, W8{});
  } else {
    if (slots_dtype == XENCB_F16) rc = read_softmax ? run(F16T{}, ST{}, W16{}) : run(F16T{}, SF{}, W16{});
    else rc = read_softmax ? run(BF16T{}, ST{}, W16{}) : run(BF16T{}, SF{}, W16{});
  }
  return rc;
}

int xencb_route_lse(const float* q, int64_t n_rows, int d_s, const float* S, int n_chunks, const int32_t* n_chunks_of,
                    int64_t rows_per_lib, int64_t n_lib, float route_temp, float* w_out, float* header_out,
                    void* stream) {
  if (!q || !S || !w_out || !header_out) return fail(XENCB_EINVAL, "route_lse: q, S, w_out and header_out are required");
  if (n_rows <= 0 || d_s <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0)
    return fail(XENCB_EINVAL, "route_lse: sizes must be positive");
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "route_lse: %lld rows need more than %lld Libraries", (long long)n_rows, (long long)n_lib);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc_t rl = launch_route_logits(q, n_rows, d_s, S, n_chunks, n_chunks_of, rows_per_lib, route_temp, w_out, st);
  if (rl) return rl;
  route_lse_kernel<<<(unsigned)((n_rows + 3) / 4), 128, 0, st>>>(w_out, n_rows, n_chunks, n_chunks_of, rows_per_lib,
                                                                 header_out);
  XENCB_CHECK_LAUNCH("route_lse launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ peer exchange
size_t xencb_exch_bytes(int world, int64_t per) {
  if (world <= 0 || world > EX_MAX_RANKS || per <= 0) return 0;
  return align_up((size_t)EX_FLAG_BYTES + 2 * (size_t)world * (size_t)per * sizeof(float), 256);
}

int xencb_exch_alloc(size_t bytes, void** ptr, void* handle_out) {
  if (!ptr || !handle_out || bytes == 0) return fail(XENCB_EINVAL, "exch_alloc: ptr, handle_out and bytes are required");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(XENCB_ECUDA, "exch_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(XENCB_ECUDA, "exch_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return XENCB_OK;
}

int xencb_exch_open(const void* handle, void** peer_ptr) {
  if (!handle || !peer_ptr) return fail(XENCB_EINVAL, "exch_open: handle and peer_ptr are required");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(XENCB_ECUDA, "exch_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *peer_ptr = p;
  return XENCB_OK;
}

int xencb_exch_close(void* peer_ptr) {
  if (!peer_ptr) return XENCB_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  if (e != cudaSuccess) return fail(XENCB_ECUDA, "exch_close: %s", cudaGetErrorString(e));
  return XENCB_OK;
}

int xencb_exch_free(void* ptr) {
  if (!ptr) return XENCB_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(XENCB_ECUDA, "exch_free: %s", cudaGetErrorString(e));
  return XENCB_OK;
}

int xencb_shard_push(const float* block, int64_t per, const void* peers_dev, int world, int rank, uint32_t* state,
                     void* stream) {
  if (!block || !peers_dev || !state) return fail(XENCB_EINVAL, "shard_push: block, peers_dev and state are required");
  if (world <= 0 || world > EX_MAX_RANKS || rank < 0 || rank >= world || per <= 0)
    return fail(XENCB_EINVAL, "shard_push: world=%d rank=%d per=%lld (1 <= world <= %d)", world, rank, (long long)per,
                EX_MAX_RANKS);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  shard_push_kernel<<<dim3((unsigned)world, EX_SLICES), EX_PUSH_THREADS, 0, st>>>(
      block, per, static_cast<const uint64_t*>(peers_dev), world, rank, state);
  XENCB_CHECK_LAUNCH("shard_push launch");
  return XENCB_OK;
}

int xencb_shard_merge_wait(const void* exch, int world, int64_t n_rows, int d_s, const uint32_t* state, float* r_out,
                           void* stream) {
  if (!exch || !state || !r_out) return fail(XENCB_EINVAL, "shard_merge_wait: exch, state and r_out are required");
  if (world <= 0 || world > EX_MAX_RANKS || n_rows <= 0 || d_s <= 0)
    return fail(XENCB_EINVAL, "shard_merge_wait: sizes must be positive (world <= %d)", EX_MAX_RANKS);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)n_rows, (unsigned)((d_s + 1023) / 1024));
  shard_merge_wait_kernel<<<grid, 256, 0, st>>>(static_cast<const char*>(exch), world, n_rows, d_s, state, r_out);
  XENCB_CHECK_LAUNCH("shard_merge_wait launch");
  return XENCB_OK;
}

int xencb_shard_merge(const float* parts, int n_shards, int64_t n_rows, int d_s, float* r_out, void* stream) {
  if (!parts || !r_out) return fail(XENCB_EINVAL, "shard_merge: parts and r_out are required");
  if (n_shards <= 0 || n_rows <= 0 || d_s <= 0) return fail(XENCB_EINVAL, "shard_merge: sizes must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)n_rows, (unsigned)((d_s + 1023) / 1024));
  shard_merge_kernel<<<grid, 256, 0, st>>>(parts, n_shards, n_rows, d_s, r_out);
  XENCB_CHECK_LAUNCH("shard_merge launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ read_prefill
size_t xencb_read_prefill_workspace(int64_t n_rows, int n_chunks, int d_s, int page_rows) {
  if (n_rows <= 0 || n_chunks <= 0 || d_s <= 0 || page_rows <= 0) return 0;
  const int64_t ncol = (page_rows + 63) / 64 * 64;
  return align_up((size_t)n_rows * d_s * 2, 256) + align_up((size_t)n_rows * n_chunks * ncol * 2, 256);
}

int xencb_read_prefill(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                       int64_t n_pages,
                       int64_t page_stride, int page_rows, const int32_t* page_of, const int32_t* n_valid, int n_chunks,
                       const int32_t* n_chunks_of, int64_t rows_per_lib, int64_t n_lib, const float* w, float read_temp,
                       int read_softmax, float* r_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !slots || !page_of || !n_valid || !w || !r_out)
    return fail(XENCB_EINVAL, "read_prefill: q, slots, page_of, n_valid, w and r_out are required");
  if (n_rows <= 0 || d_s <= 0 || page_rows <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0 || n_pages <= 0)
    return fail(XENCB_EINVAL, "read_prefill: sizes must be positive");
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "read_prefill: %lld rows need more than %lld Libraries", (long long)n_rows,
                (long long)n_lib);
  if (slots_dtype != XENCB_F16) return fail(XENCB_ENOTSUP, "read_prefill: the tensor-core prefill reads f16 slots");
  if (d_s % 64 != 0) return fail(XENCB_ENOTSUP, "read_prefill: d_s=%d must be a multiple of 64", d_s);
  if (page_rows > 512) return fail(XENCB_ENOTSUP, "read_prefill: page_rows=%d above 512", page_rows);
  if (page_stride != (int64_t)page_rows * d_s)
    return fail(XENCB_ENOTSUP, "read_prefill: the slot pool must be dense ([pages, page_rows, d_s])");
  if (n_pages * (int64_t)page_rows + 512 > INT32_MAX || (int64_t)n_chunks * 512 > INT32_MAX)
    return fail(XENCB_ENOTSUP, "read_prefill: the slot pool is too large for 32-bit TMA coordinates");
  if (!aligned(slots, 16) || !aligned(q, 16) || !aligned(r_out, 16) || (vslots && !aligned(vslots, 16)))
    return fail(XENCB_EINVAL, "read_prefill: slots, vslots, q and r_out must be 16-byte aligned");
  const size_t need = xencb_read_prefill_workspace(n_rows, n_chunks, d_s, page_rows);
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < need)
    return fail(XENCB_EINVAL, "read_prefill: workspace needs %zu bytes, 256-byte aligned (got %zu)", need,
                workspace_bytes);
  PrefillArgs a;
  a.n_rows = n_rows; a.rows_per_lib = rows_per_lib; a.d_s = d_s; a.n_chunks = n_chunks; a.page_rows = page_rows;
  a.ncol = (page_rows + 63) / 64 * 64; a.n_pages = n_pages; a.page_of = page_of; a.n_valid = n_valid;
  a.n_chunks_of = n_chunks_of; a.w = w; a.qscale = read_temp * 1.4426950408889634f; a.softmax = read_softmax ? 1 : 0;
  char* ws = static_cast<char*>(workspace);
  __half* q16 = reinterpret_cast<__half*>(ws);
  a.P = reinterpret_cast<__half*>(ws + align_up((size_t)n_rows * d_s * 2, 256));
  a.r_out = r_out;
  const int b_box_rows = a.ncol < 256 ? a.ncol : 256;
  CUtensorMap mq, mk1, mp, mk2;
  int rc = tensor_map_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, q16, (uint64_t)d_s, (uint64_t)n_rows,
                         (uint64_t)d_s * 2, PF_S_BK, PF_BM, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc) rc = tensor_map_2d(&mk1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, slots, (uint64_t)d_s,
                              (uint64_t)(n_pages * page_rows), (uint64_t)d_s * 2, PF_S_BK, (uint32_t)b_box_rows,
                              CU_TENSOR_MAP_SWIZZLE_64B);
  if (!rc) rc = tensor_map_2d(&mp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.P, (uint64_t)n_chunks * a.ncol,
                              (uint64_t)n_rows, (uint64_t)n_chunks * a.ncol * 2, PF_BK, PF_BM);
  if (!rc) rc = tensor_map_2d(&mk2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, vslots ? vslots : slots, (uint64_t)d_s,
                              (uint64_t)(n_pages * page_rows), (uint64_t)d_s * 2, 64, PF_BK);
  if (rc) return rc;
  rc = ensure_smem(prefill_scores_kernel, (int)PF_S_SMEM);
  if (!rc) rc = ensure_smem(prefill_read_kernel, (int)PF_R_SMEM);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t nq = n_rows * (int64_t)d_s;
  to_f16_kernel<<<(unsigned)std::min<int64_t>((nq / 4 + 255) / 256, 8192), 256, 0, st>>>(q, nq, q16);
  XENCB_CHECK_LAUNCH("to_f16 launch");
  const int64_t libs_used = (n_rows + rows_per_lib - 1) / rows_per_lib;
  const unsigned tiles = (unsigned)((rows_per_lib + PF_BM - 1) / PF_BM);
  prefill_scores_kernel<<<dim3(tiles, (unsigned)n_chunks, (unsigned)libs_used), PF_S_THREADS, PF_S_SMEM, st>>>(
      mq, mk1, mp, a, b_box_rows);
  XENCB_CHECK_LAUNCH("prefill_scores launch");
  // d_s in 512-column slices: the read as CTA pairs (half the operand bytes per SM); XENCB_PREFILL_PAIR=0 in the
  // environment keeps the single-CTA kernel
  const char* pair_env = getenv("XENCB_PREFILL_PAIR");
  if (d_s % PF2R_BN == 0 && !(pair_env && pair_env[0] == '0')) {
    rc = ensure_smem(prefill_read_pair_kernel, (int)PF2R_SMEM);
    if (rc) return rc;
    prefill_read_pair_kernel<<<dim3((tiles + 1) / 2 * 2, (unsigned)(d_s / PF2R_BN), (unsigned)libs_used),
                               PF_THREADS, PF2R_SMEM, st>>>(mp, mk2, a);
  } else {
    prefill_read_kernel<<<dim3(tiles, (unsigned)((d_s + PF_R_BN - 1) / PF_R_BN), (unsigned)libs_used), PF_THREADS,
                          PF_R_SMEM, st>>>(mp, mk2, a);
  }
  XENCB_CHECK_LAUNCH("prefill_read launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ project_out
size_t xencb_project_out_workspace(int64_t n_rows, int d_s, int d_m) {
  DevInfo di;
  if (device_info(&di)) return 0;
  if (n_rows <= 0 || d_m <= 0 || d_s <= 0) return 0;
  const int nch = (d_m + PIN_CHUNK - 1) / PIN_CHUNK;
  return gemm_ws_bytes(n_rows, d_m, d_s, di.sms, false) + align_up((size_t)n_rows * d_m * sizeof(float), 256) +
         align_up((size_t)n_rows * nch * 3 * sizeof(float), 256) + align_up((size_t)n_rows * sizeof(int), 256);
}

int xencb_project_out(const float* r, int64_t n_rows, int d_s, const float* w_out, const void* w_prep,
                      const float* b_out, int d_m,
                      float scale, const float* log_scale_dev, const float* gate, const float* sel_w, float log_alpha,
                      const float* log_alpha_dev, const float* pos_mask,
                      const void* h, int h_dtype, void* delta_out, void* h_out, float* rel_out, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (!r || (!w_out && !w_prep) || !h) return fail(XENCB_EINVAL, "project_out: r, w_out (or w_prep) and h are required");
  if (!w_out && (d_s % 8 != 0 || !aligned(w_prep, 256)))
    return fail(XENCB_EINVAL, "project_out: without w_out, w_prep must be 256-byte aligned and d_s %% 8 == 0");
  if (n_rows <= 0 || d_m <= 0 || d_s <= 0) return fail(XENCB_EINVAL, "project_out: sizes must be positive");
  if (!elem_size(h_dtype)) return fail(XENCB_EINVAL, "project_out: h_dtype %d unknown", h_dtype);
  if (d_m % 4 != 0)
    return fail(XENCB_EINVAL, "project_out: d_m=%d must be a multiple of 4", d_m);
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int nch = (d_m + PIN_CHUNK - 1) / PIN_CHUNK;
  const size_t g_bytes = gemm_ws_bytes(n_rows, d_m, d_s, di.sms, false);
  const size_t d_bytes = align_up((size_t)n_rows * d_m * sizeof(float), 256);
  const size_t np_bytes = align_up((size_t)n_rows * nch * 3 * sizeof(float), 256);
  const size_t need = g_bytes + d_bytes + np_bytes + align_up((size_t)n_rows * sizeof(int), 256);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(XENCB_EINVAL, "project_out: workspace needs %zu bytes, 256-byte aligned (got %zu)", need,
                workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  float* part = reinterpret_cast<float*>(ws);
  float* dbuf = reinterpret_cast<float*>(ws + g_bytes);
  float* norm_part = reinterpret_cast<float*>(ws + g_bytes + d_bytes);
  float* cn_part = norm_part + (size_t)n_rows * nch * 2;
  int* row_done = reinterpret_cast<int*>(ws + g_bytes + d_bytes + np_bytes);
  GemmPlan gp;
  float* xbuf = (d_s % 4 == 0) ? reinterpret_cast<float*>(ws + gemm_part_bytes(n_rows, d_m, d_s, di.sms)) : nullptr;
  rc = launch_gemm<float>(r, n_rows, d_s, w_out, d_m, di.sms, part, w_prep ? xbuf : nullptr, nullptr, st, &gp, w_prep);
  if (rc) return rc;
  const float alpha = expf(log_alpha);
  if (d_m <= 12 * ROW_THREADS) {  // one CTA per row: the reduce, the norms and the epilogue in registers
    const int vpt = (d_m + 4 * ROW_THREADS - 1) / (4 * ROW_THREADS);  // float4 columns per thread: 1..3
    const unsigned thr = (unsigned)std::min<int>(ROW_THREADS, (d_m / 4 + 31) / 32 * 32);
    auto launch = [&](auto kern, auto* hp) {
      launch_pdl(kern, dim3((unsigned)n_rows), dim3(thr), 0, st, part, gp.splits, n_rows, d_m, b_out, scale,
                 log_scale_dev, gate, hp, sel_w, alpha, log_alpha_dev, pos_mask,
                 static_cast<decltype(hp)>(delta_out), static_cast<decltype(hp)>(h_out), rel_out);
    };
    auto by_vpt = [&](auto* hp) {
      using TH = std::remove_pointer_t<decltype(hp)>;
      if (vpt == 1) launch(project_out_row_kernel<TH, 1>, hp);
      else if (vpt == 2) launch(project_out_row_kernel<TH, 2>, hp);
      else launch(project_out_row_kernel<TH, 3>, hp);
    };
    switch (h_dtype) {
      case XENCB_F32: by_vpt(static_cast<float*>(const_cast<void*>(h))); break;
      case XENCB_F16: by_vpt(static_cast<__half*>(const_cast<void*>(h))); break;
      default: by_vpt(static_cast<__nv_bfloat16*>(const_cast<void*>(h))); break;
    }
    XENCB_CHECK_LAUNCH("project_out row launch");
    return XENCB_OK;
  }
#define XENCB_POUT(T)                                                                                          \
  do {                                                                                                         \
    project_out_reduce_kernel<T><<<dim3((unsigned)n_rows, nch), 256, 0, st>>>(                                \
        part, gp.splits, n_rows, d_m, b_out, scale, log_scale_dev, gate, static_cast<const T*>(h), dbuf,       \
        norm_part, row_done);                                                                                  \
    project_out_epilogue_kernel<T><<<dim3((unsigned)n_rows, nch), 256, 0, st>>>(                               \
        dbuf, norm_part, d_m, sel_w, alpha, log_alpha_dev, pos_mask, static_cast<const T*>(h),                 \
        static_cast<T*>(delta_out),                                                                            \
        static_cast<T*>(h_out), rel_out, cn_part, row_done);                                                   \
  } while (0)
  switch (h_dtype) {
    case XENCB_F32: XENCB_POUT(float); break;
    case XENCB_F16: XENCB_POUT(__half); break;
    default: XENCB_POUT(__nv_bfloat16); break;
  }
#undef XENCB_POUT
  XENCB_CHECK_LAUNCH_N("project_out reduce + epilogue launch", 2);
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ selector
int xencb_selector_weights(const float* z, int64_t n_rows, int n_cand, int k, int straight_through, float* w_out,
                           void* stream) {
  if (!z || !w_out) return fail(XENCB_EINVAL, "selector_weights: z and w_out are required");
  if (n_rows <= 0 || n_cand <= 0 || n_cand > 32)
    return fail(XENCB_EINVAL, "selector_weights: need n_rows > 0 and 1 <= n_cand <= 32 (got %d)", n_cand);
  if (k < 1 || k > n_cand) return fail(XENCB_EINVAL, "k=%d must be in [1, %d]", k, n_cand);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  selector_weights_kernel<<<(unsigned)((n_rows + 3) / 4), 128, 0, st>>>(z, n_rows, n_cand, k, straight_through,
                                                                          w_out);
  XENCB_CHECK_LAUNCH("selector_weights launch");
  return XENCB_OK;
}

int xencb_selector_logits(const void* h, int h_dtype, int64_t n_rows, int d_m, const float* u_w, const float* u_b,
                          int n_cand, int rms, float rms_eps, float* z_out, void* stream) {
  if (!h || !u_w || !z_out) return fail(XENCB_EINVAL, "selector_logits: h, u_w and z_out are required");
  if (n_rows <= 0 || d_m <= 0 || n_cand <= 0 || n_cand > 32)
    return fail(XENCB_EINVAL, "selector_logits: need positive sizes and n_cand <= 32 (got %d)", n_cand);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (h_dtype) {
    case XENCB_F32:
      selector_logits_kernel<float><<<(unsigned)n_rows, 256, 0, st>>>(static_cast<const float*>(h), d_m, u_w, u_b,
                                                                       n_cand, rms, rms_eps, z_out);
      break;
    case XENCB_F16:
      selector_logits_kernel<__half><<<(unsigned)n_rows, 256, 0, st>>>(static_cast<const __half*>(h), d_m, u_w, u_b,
                                                                        n_cand, rms, rms_eps, z_out);
      break;
    case XENCB_BF16:
      selector_logits_kernel<__nv_bfloat16><<<(unsigned)n_rows, 256, 0, st>>>(
          static_cast<const __nv_bfloat16*>(h), d_m, u_w, u_b, n_cand, rms, rms_eps, z_out);
      break;
    default: return fail(XENCB_EINVAL, "selector_logits: h_dtype %d unknown", h_dtype);
  }
  XENCB_CHECK_LAUNCH("selector_logits launch");
  return XENCB_OK;
}

int xencb_selector_apply(const void* delta, int delta_dtype, const void* h, int h_dtype, int64_t n_rows, int d,
                         const float* w, int n_cand, int pos, float log_alpha, void* out, void* stream) {
  if (!delta || !h || !w || !out) return fail(XENCB_EINVAL, "selector_apply: null pointer argument");
  if (n_rows <= 0 || d <= 0 || n_cand <= 0 || pos < 0 || pos >= n_cand)
    return fail(XENCB_EINVAL, "selector_apply: bad sizes (n_rows=%lld d=%d n_cand=%d pos=%d)", (long long)n_rows, d,
                n_cand, pos);
  if (!elem_size(delta_dtype) || !elem_size(h_dtype)) return fail(XENCB_EINVAL, "selector_apply: unknown dtype");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float alpha = expf(log_alpha);
  switch (delta_dtype) {
    case XENCB_F32: launch_sel_apply<float>(delta, h, h_dtype, n_rows, d, w, n_cand, pos, alpha, out, st); break;
    case XENCB_F16: launch_sel_apply<__half>(delta, h, h_dtype, n_rows, d, w, n_cand, pos, alpha, out, st); break;
    default: launch_sel_apply<__nv_bfloat16>(delta, h, h_dtype, n_rows, d, w, n_cand, pos, alpha, out, st); break;
  }
  XENCB_CHECK_LAUNCH("selector_apply launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ summaries
int xencb_summaries(const void* slots, int slots_dtype, int64_t n_pages, int64_t page_stride, int page_rows,
                    const int32_t* page_of,
                    const int32_t* n_valid, int64_t n_lib, int n_chunks, int d_s, float* S_out, void* stream) {
  if (!slots || !page_of || !n_valid || !S_out) return fail(XENCB_EINVAL, "summaries: null pointer argument");
  if (n_lib <= 0 || n_chunks <= 0 || d_s <= 0 || page_rows <= 0 || n_pages <= 0)
    return fail(XENCB_EINVAL, "summaries: sizes must be positive");
  if (page_stride < (int64_t)page_rows * d_s) return fail(XENCB_EINVAL, "summaries: page_stride too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)(n_lib * n_chunks);
  switch (slots_dtype) {
    case XENCB_F32:
      summaries_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(slots), n_pages, page_stride, page_rows,
                                                      page_of, n_valid, n_chunks, d_s, S_out);
      break;
    case XENCB_F16:
      summaries_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(slots), n_pages, page_stride, page_rows,
                                                       page_of, n_valid, n_chunks, d_s, S_out);
      break;
    case XENCB_BF16:
      summaries_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(slots), n_pages, page_stride,
                                                              page_rows, page_of, n_valid, n_chunks, d_s, S_out);
      break;
    default: return fail(XENCB_EINVAL, "summaries: slots_dtype %d unknown", slots_dtype);
  }
  XENCB_CHECK_LAUNCH("summaries launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ library build

size_t xencb_library_build_workspace(int n_chunks, int d_s, int page_rows) {
  if (n_chunks <= 0 || d_s <= 0 || page_rows <= 0) return 0;
  BuildPlan p;
  if (plan_build(n_chunks, d_s, page_rows, &p)) return 0;
  return p.part_bytes;
}

int xencb_library_build(const void* rows, int rows_dtype, int64_t n_rows_total, const int64_t* row_start, int n_chunks,
                        int d_s, const float* mu, void* slots, int slots_dtype, int64_t n_pages, int64_t page_stride,
                        int page_rows, const int32_t* page_of, int32_t* n_valid_out, float* S_out, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!row_start || !slots || !page_of) return fail(XENCB_EINVAL, "library_build: row_start, slots and page_of are required");
  if (n_rows_total < 0 || (n_rows_total > 0 && !rows)) return fail(XENCB_EINVAL, "library_build: rows is required");
  if (n_chunks <= 0 || d_s <= 0 || page_rows <= 0 || n_pages <= 0)
    return fail(XENCB_EINVAL, "library_build: sizes must be positive");
  if (d_s % LB_VEC) return fail(XENCB_EINVAL, "library_build: d_s=%d must be a multiple of %d", d_s, LB_VEC);
  const int ei = elem_size(rows_dtype), eo = elem_size(slots_dtype);
  if (!ei || !eo) return fail(XENCB_EINVAL, "library_build: dtype codes %d / %d unknown", rows_dtype, slots_dtype);
  if (page_stride < (int64_t)page_rows * d_s)
    return fail(XENCB_EINVAL, "library_build: page_stride %lld < page_rows*d_s %lld", (long long)page_stride,
                (long long)page_rows * d_s);
  if ((rows && !aligned(rows, 16)) || !aligned(slots, 16) || (page_stride * eo) % 16 != 0 || (mu && !aligned(mu, 16)))
    return fail(XENCB_EINVAL, "library_build: rows, slots, mu and page_stride*elem must be 16-byte aligned");
  BuildPlan p;
  int rc = plan_build(n_chunks, d_s, page_rows, &p);
  if (rc) return rc;
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < p.part_bytes)
    return fail(XENCB_EINVAL, "library_build: workspace needs %zu bytes, 256-byte aligned (got %zu)", p.part_bytes,
                workspace_bytes);
  LibBuildArgs a;
  a.rows = rows; a.n_rows_total = n_rows_total; a.row_start = row_start; a.n_chunks = n_chunks; a.d_s = d_s;
  a.mu = mu; a.slots = slots; a.n_pages = n_pages; a.page_stride = page_stride; a.page_rows = page_rows;
  a.page_of = page_of; a.n_split = p.n_split; a.split_rows = p.split_rows;
  a.part = static_cast<float*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto run = [&](auto ti, auto to) -> int {
    using TI = typename decltype(ti)::type;
    using TO = typename decltype(to)::type;
    library_build_kernel<TI, TO><<<dim3((unsigned)n_chunks, (unsigned)p.n_split), p.threads, 0, st>>>(a);
    XENCB_CHECK_LAUNCH("library_build_kernel launch");
    library_summaries_kernel<<<(unsigned)n_chunks, 256, 0, st>>>(a, n_valid_out, S_out);
    XENCB_CHECK_LAUNCH("library_summaries_kernel launch");
    return XENCB_OK;
  };
  struct F32T { using type = float; };
  struct F16T { using type = __half; };
  struct BF16T { using type = __nv_bfloat16; };
  auto with_out = [&](auto ti) -> int {
    switch (slots_dtype) {
      case XENCB_F32: return run(ti, F32T{});
      case XENCB_F16: return run(ti, F16T{});
      default: return run(ti, BF16T{});
    }
  };
  switch (rows_dtype) {
    case XENCB_F32: return with_out(F32T{});
    case XENCB_F16: return with_out(F16T{});
    default: return with_out(BF16T{});
  }
}

// ------------------------------------------------------------------------------------------------ D8 top-k read
int xencb_select_scores(const float* q, int64_t n_rows, int T, int n_q, int n_kv, int hd, const void* keys,
                        int keys_dtype, int64_t keys_lib_stride, int page_rows, int n_chunks, const int32_t* n_valid,
                        const int32_t* n_chunks_of, int64_t rows_per_lib, int64_t n_lib, int query_pool, int head_pool,
                        float* scores_out, void* stream) {
  if (!q || !keys || !n_valid || !scores_out) return fail(XENCB_EINVAL, "select_scores: null pointer argument");
  if (n_rows <= 0 || T <= 0 || n_q <= 0 || n_kv <= 0 || hd <= 0 || page_rows <= 0 || n_chunks <= 0 ||
      rows_per_lib <= 0 || n_lib <= 0)
    return fail(XENCB_EINVAL, "select_scores: sizes must be positive");
  if (n_q % n_kv) return fail(XENCB_EINVAL, "select_scores: n_q=%d is not a multiple of n_kv=%d", n_q, n_kv);
  if (n_q / n_kv > SEL_MAX_G || n_kv > SEL_MAX_KV)
    return fail(XENCB_ENOTSUP, "select_scores: GQA groups <= %d and n_kv <= %d are supported", SEL_MAX_G, SEL_MAX_KV);
  if (hd % 8) return fail(XENCB_EINVAL, "select_scores: head_dim=%d must be a multiple of 8", hd);
  if ((n_rows + rows_per_lib - 1) / rows_per_lib > n_lib)
    return fail(XENCB_EINVAL, "select_scores: %lld rows need more than %lld Libraries", (long long)n_rows,
                (long long)n_lib);
  if (query_pool < 0 || query_pool > 1 || head_pool < 0 || head_pool > 1)
    return fail(XENCB_EINVAL, "select_scores: query_pool / head_pool must be 0 (max) or 1 (mean)");
  if ((int64_t)n_chunks * page_rows > INT32_MAX) return fail(XENCB_EINVAL, "select_scores: too many slots");
  const int es = elem_size(keys_dtype);
  if (keys_dtype != XENCB_F32 && keys_dtype != XENCB_F16)
    return fail(XENCB_EINVAL, "select_scores: keys must be XENCB_F32 or XENCB_F16");
  if (keys_lib_stride < (int64_t)n_chunks * page_rows * n_kv * hd && n_lib > 1)
    return fail(XENCB_EINVAL, "select_scores: keys_lib_stride smaller than one Library's keys");
  if (!aligned(q, 16) || !aligned(keys, 16) || (keys_lib_stride * es) % 16)
    return fail(XENCB_EINVAL, "select_scores: q, keys and keys_lib_stride*elem must be 16-byte aligned");
  SelectArgs a;
  a.q = q; a.n_rows = n_rows; a.T = T; a.n_q = n_q; a.n_kv = n_kv; a.hd = hd; a.keys = keys;
  a.keys_lib_stride = keys_lib_stride; a.page_rows = page_rows; a.n_chunks = n_chunks; a.n_valid = n_valid;
  a.n_chunks_of = n_chunks_of; a.rows_per_lib = rows_per_lib; a.t_pool = query_pool; a.h_pool = head_pool;
  a.scores = scores_out;
  const int S = n_chunks * page_rows;
  dim3 grid((unsigned)((S + SEL_TILE - 1) / SEL_TILE), (unsigned)n_rows);
  if (n_rows > 65535) return fail(XENCB_ENOTSUP, "select_scores: at most 65535 rows per call");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // one position with f16 keys: the tensor-core scores (XENCB_SELECT_SIMT=1 in the environment keeps the FMA path)
  const int G = n_q / n_kv;
  const char* simt = getenv("XENCB_SELECT_SIMT");
  if (T == 1 && keys_dtype == XENCB_F16 && (G == 1 || G == 2 || G == 4) &&
      (hd == 32 || hd == 64 || hd == 128) && !(simt && simt[0] == '1')) {
    auto by_p2 = [&](auto k1, auto k2, auto k4) {
      switch (hd) {
        case 32: k1<<<grid, SEL_THREADS, 0, st>>>(a); break;
        case 64: k2<<<grid, SEL_THREADS, 0, st>>>(a); break;
        default: k4<<<grid, SEL_THREADS, 0, st>>>(a); break;
      }
    };
#define XENCB_SELM(GG) \
  by_p2(select_scores_mma_kernel<GG, 1>, select_scores_mma_kernel<GG, 2>, select_scores_mma_kernel<GG, 4>)
    if (G == 1) XENCB_SELM(1);
    else if (G == 2) XENCB_SELM(2);
    else XENCB_SELM(4);
#undef XENCB_SELM
    XENCB_CHECK_LAUNCH("select_scores_mma_kernel launch");
    return XENCB_OK;
  }
  auto run = [&](auto kf, auto kh) {
    if (keys_dtype == XENCB_F32) kf<<<grid, SEL_THREADS, 0, st>>>(a);
    else kh<<<grid, SEL_THREADS, 0, st>>>(a);
  };
  switch (n_q / n_kv) {
    case 1: run(select_scores_kernel<float, 1>, select_scores_kernel<__half, 1>); break;
    case 2: run(select_scores_kernel<float, 2>, select_scores_kernel<__half, 2>); break;
    case 4: run(select_scores_kernel<float, 4>, select_scores_kernel<__half, 4>); break;
    case 8: run(select_scores_kernel<float, 8>, select_scores_kernel<__half, 8>); break;
    case 16: run(select_scores_kernel<float, 16>, select_scores_kernel<__half, 16>); break;
    default: return fail(XENCB_ENOTSUP, "select_scores: GQA group %d (supported: 1, 2, 4, 8, 16)", n_q / n_kv);
  }
  XENCB_CHECK_LAUNCH("select_scores_kernel launch");
  return XENCB_OK;
}

int xencb_select_topk(const float* scores, int64_t n_rows, int n_slots, int k, int32_t* idx_out, float* score_out,
                      void* stream) {
  if (!scores || !idx_out) return fail(XENCB_EINVAL, "select_topk: scores and idx_out are required");
  if (n_rows <= 0 || n_slots <= 0 || k <= 0) return fail(XENCB_EINVAL, "select_topk: sizes must be positive");
  if (k > n_slots) return fail(XENCB_EINVAL, "select_topk: k=%d > %d slots", k, n_slots);
  if (k > TOPK_MAX_K) return fail(XENCB_ENOTSUP, "select_topk: k=%d above %d is not supported", k, TOPK_MAX_K);
  if (n_rows > INT32_MAX) return fail(XENCB_EINVAL, "select_topk: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // rows up to 32,768 slots: a cluster of 8 CTAs per row; XENCB_TOPK_CLUSTER=0 in the environment keeps one CTA
  const char* cl_env = getenv("XENCB_TOPK_CLUSTER");
  if (n_slots <= TKC_CL * TKC_THREADS * TKC_KPT && n_rows * TKC_CL <= INT32_MAX && !(cl_env && cl_env[0] == '0'))
    select_topk_cluster_kernel<<<(unsigned)(n_rows * TKC_CL), TKC_THREADS, 0, st>>>(scores, n_slots, k, idx_out,
                                                                                    score_out);
  else
    select_topk_kernel<<<(unsigned)n_rows, TOPK_THREADS, 0, st>>>(scores, n_slots, k, idx_out, score_out);
  XENCB_CHECK_LAUNCH("select_topk_kernel launch");
  return XENCB_OK;
}

int xencb_topk_read(const float* q, int64_t n_rows, int d_s, const void* slots, const void* vslots, int slots_dtype,
                    int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of, int n_chunks,
                    int64_t n_lib, const int32_t* idx, int n_sets, int k, float read_temp, int read_softmax,
                    float* r_out, float* attn_out, void* stream) {
  if (!q || !slots || !page_of || !idx || !r_out) return fail(XENCB_EINVAL, "topk_read: null pointer argument");
  if (n_rows <= 0 || d_s <= 0 || n_pages <= 0 || page_rows <= 0 || n_chunks <= 0 || n_lib <= 0 || n_sets <= 0 ||
      k <= 0)
    return fail(XENCB_EINVAL, "topk_read: sizes must be positive");
  if (n_rows % n_sets) return fail(XENCB_EINVAL, "topk_read: %lld rows are not a multiple of %d index sets",
                                   (long long)n_rows, n_sets);
  if (n_lib > 1 && n_lib != n_sets)
    return fail(XENCB_EINVAL, "topk_read: %lld Libraries need one index set each (got %d)", (long long)n_lib, n_sets);
  if (d_s % 8) return fail(XENCB_EINVAL, "topk_read: d_s=%d must be a multiple of 8", d_s);
  const int es = elem_size(slots_dtype);
  if (!es) return fail(XENCB_EINVAL, "topk_read: slots_dtype %d unknown", slots_dtype);
  if (page_stride < (int64_t)page_rows * d_s) return fail(XENCB_EINVAL, "topk_read: page_stride too small");
  if (!aligned(q, 16) || !aligned(slots, 16) || (vslots && !aligned(vslots, 16)) || !aligned(r_out, 16) ||
      (page_stride * es) % 16)
    return fail(XENCB_EINVAL, "topk_read: q, slots, vslots, r_out and page_stride*elem must be 16-byte aligned");
  const int nt_cta = n_rows / n_sets == 1 ? 1 : TR_ROWS;  // decode (one row per set): no work for absent rows
  if (nt_cta == 1) {
    // decode: a 4-CTA cluster per set (k split over the cluster, combined through distributed shared memory)
    const int per = (k + TRC - 1) / TRC;
    const size_t dsm = (2 * (size_t)d_s + (((size_t)per + 3) & ~(size_t)3) + 4) * sizeof(float) +
                       (size_t)per * sizeof(int64_t);
    if ((int64_t)n_sets * TRC > INT32_MAX) return fail(XENCB_EINVAL, "topk_read: too many index sets");
    TopkReadArgs d;
    d.q = q; d.n_rows = n_rows; d.d_s = d_s;
    d.slots = static_cast<const char*>(slots);
    d.vslots = static_cast<const char*>(vslots);
    d.n_pages = n_pages; d.page_stride_bytes = page_stride * es; d.page_rows = page_rows; d.n_chunks = n_chunks;
    d.page_of = page_of; d.n_lib = n_lib; d.idx = idx; d.n_sets = n_sets; d.k = k; d.rows_per_set = 1;
    d.qscale = read_softmax ? read_temp * 1.4426950408889634f : 1.f;
    d.softmax = read_softmax ? 1 : 0;
    d.r_out = r_out; d.attn_out = attn_out;
    cudaStream_t st0 = static_cast<cudaStream_t>(stream);
    auto launch_d = [&](auto kern) -> int {
      int r2 = ensure_smem(kern, (int)dsm);
      if (r2) return r2;
      kern<<<(unsigned)(n_sets * TRC), TR_THREADS, dsm, st0>>>(d);
      XENCB_CHECK_LAUNCH("topk_read_decode_kernel launch");
      return XENCB_OK;
    };
    switch (slots_dtype) {
      case XENCB_F32: return launch_d(topk_read_decode_kernel<float>);
      case XENCB_F16: return launch_d(topk_read_decode_kernel<__half>);
      default: return launch_d(topk_read_decode_kernel<__nv_bfloat16>);
    }
  }
  const size_t smem = ((size_t)nt_cta * d_s + (((size_t)nt_cta * k + 1) & ~(size_t)1)) * sizeof(float) +
                      (size_t)k * sizeof(int64_t);
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (smem > (size_t)(di.max_smem_optin > 0 ? di.max_smem_optin : 232448))
    return fail(XENCB_ENOTSUP, "topk_read: d_s=%d with k=%d does not fit in shared memory", d_s, k);
  TopkReadArgs a;
  a.q = q; a.n_rows = n_rows; a.d_s = d_s;
  a.slots = static_cast<const char*>(slots);
  a.vslots = static_cast<const char*>(vslots);
  a.n_pages = n_pages; a.page_stride_bytes = page_stride * es; a.page_rows = page_rows; a.n_chunks = n_chunks;
  a.page_of = page_of; a.n_lib = n_lib; a.idx = idx; a.n_sets = n_sets; a.k = k;
  a.rows_per_set = n_rows / n_sets;
  a.qscale = read_softmax ? read_temp * 1.4426950408889634f : 1.f;
  a.softmax = read_softmax ? 1 : 0;
  a.r_out = r_out; a.attn_out = attn_out;
  const int64_t yblocks = (a.rows_per_set + nt_cta - 1) / nt_cta;
  if (yblocks > 65535) return fail(XENCB_ENOTSUP, "topk_read: too many rows per index set");
  dim3 grid((unsigned)n_sets, (unsigned)yblocks);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kern) -> int {
    int r2 = ensure_smem(kern, (int)smem);
    if (r2) return r2;
    kern<<<grid, TR_THREADS, smem, st>>>(a);
    XENCB_CHECK_LAUNCH("topk_read_kernel launch");
    return XENCB_OK;
  };
  if (nt_cta == 1) {
    switch (slots_dtype) {
      case XENCB_F32: return launch(topk_read_kernel<float, 1>);
      case XENCB_F16: return launch(topk_read_kernel<__half, 1>);
      default: return launch(topk_read_kernel<__nv_bfloat16, 1>);
    }
  }
  switch (slots_dtype) {
    case XENCB_F32: return launch(topk_read_kernel<float, TR_ROWS>);
    case XENCB_F16: return launch(topk_read_kernel<__half, TR_ROWS>);
    default: return launch(topk_read_kernel<__nv_bfloat16, TR_ROWS>);
  }
}

size_t xencb_weights_prep_bytes(int n, int k) {
  if (n <= 0 || k <= 0) return 0;
  return WPREP_HEAD + (size_t)wprep_pairs(n, k) * WPREP_PAIR * sizeof(__half);
}

int xencb_weights_prep(const float* w, int n, int k, void* prep, size_t prep_bytes, void* stream) {
  if (!w || !prep) return fail(XENCB_EINVAL, "weights_prep: w and prep are required");
  if (n <= 0 || k <= 0) return fail(XENCB_EINVAL, "weights_prep: sizes must be positive");
  if (k % 8) return fail(XENCB_EINVAL, "weights_prep: k=%d must be a multiple of 8", k);
  if (!aligned(prep, 256)) return fail(XENCB_EINVAL, "weights_prep: prep must be 256-byte aligned");
  if (prep_bytes < xencb_weights_prep_bytes(n, k))
    return fail(XENCB_EINVAL, "weights_prep: prep needs %zu bytes (got %zu)", xencb_weights_prep_bytes(n, k), prep_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int* head = static_cast<unsigned int*>(prep);
  cudaError_t e = cudaMemsetAsync(head, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return cuda_fail(e, "weights_prep memset");
  const int64_t cnt = (int64_t)n * k;
  const unsigned blocks = (unsigned)std::min<int64_t>((cnt + 255) / 256, 4096);
  absmax_kernel<<<blocks, 256, 0, st>>>(w, cnt, head);
  XENCB_CHECK_LAUNCH("absmax launch");
  __half* tiles = reinterpret_cast<__half*>(static_cast<char*>(prep) + WPREP_HEAD);
  split_weights_kernel<<<blocks, 256, 0, st>>>(w, n, k, head, tiles, reinterpret_cast<float*>(head) + 1);
  XENCB_CHECK_LAUNCH("split_weights launch");
  return XENCB_OK;
}

int xencb_read_kernel_events(void* before, void* after) {
  g_read_ev_before = static_cast<cudaEvent_t>(before);
  g_read_ev_after = static_cast<cudaEvent_t>(after);
  return XENCB_OK;
}

int xencb_wait_selftest(long long limit_cycles, int* result, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > 4000000000ll)
    return fail(XENCB_EINVAL, "wait_selftest: limit_cycles must be in (0, 4e9]");
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_cycles, result);
  XENCB_CHECK_LAUNCH("wait_selftest_kernel launch");
  return XENCB_OK;
}

// ------------------------------------------------------------------------------------------------ attention diagnostics
int xencb_read_attn(const float* q, int64_t row, int d_s, const void* slots, int slots_dtype, int64_t n_pages,
                    int64_t page_stride, int page_rows, const int32_t* page_of, const int32_t* n_valid, int n_chunks,
                    int64_t rows_per_lib, int64_t n_lib, const int32_t* idx, const float* wk, int k, float read_temp,
                    int read_softmax, float* attn_out, void* stream) {
  if (!q || !slots || !page_of || !n_valid || !idx || !wk || !attn_out)
    return fail(XENCB_EINVAL, "read_attn: q, slots, page_of, n_valid, idx, wk and attn_out are required");
  if (row < 0 || d_s <= 0 || page_rows <= 0 || n_chunks <= 0 || rows_per_lib <= 0 || n_lib <= 0 || k <= 0 ||
      n_pages <= 0)
    return fail(XENCB_EINVAL, "read_attn: sizes must be positive and row >= 0");
  const int64_t lib = row / rows_per_lib;
  if (lib >= n_lib) return fail(XENCB_EINVAL, "read_attn: row %lld reads Library %lld of %lld", (long long)row,
                                (long long)lib, (long long)n_lib);
  const int es = elem_size(slots_dtype);
  if (!es) return fail(XENCB_EINVAL, "read_attn: slots_dtype %d unknown", slots_dtype);
  if (page_stride < (int64_t)page_rows * d_s)
    return fail(XENCB_EINVAL, "read_attn: page_stride %lld < page_rows*d_s", (long long)page_stride);
  const size_t smem = ((size_t)d_s + (size_t)page_rows) * sizeof(float);
  if (smem > 200 * 1024) return fail(XENCB_ENOTSUP, "read_attn: d_s + page_rows = %zu floats exceed shared memory",
                                     smem / 4);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* qr = q + row * (int64_t)d_s;
  const int32_t* po = page_of + lib * n_chunks;
  const int32_t* nv = n_valid + lib * n_chunks;
  const int32_t* ir = idx + row * (int64_t)k;
  const float* wr = wk + row * (int64_t)k;
  const char* sp = static_cast<const char*>(slots);
  auto run = [&](auto kern) -> int {
    int rc = ensure_smem(kern, (int)std::max<size_t>(smem, 48 * 1024));
    if (rc) return rc;
    kern<<<(unsigned)n_chunks, AT_THREADS, smem, st>>>(qr, d_s, sp, n_pages, page_stride * es, page_rows, po, nv, ir,
                                                       wr, k, read_temp, read_softmax, attn_out);
    XENCB_CHECK_LAUNCH("read_attn launch");
    return XENCB_OK;
  };
  switch (slots_dtype) {
    case XENCB_F16: return run(read_attn_kernel<__half>);
    case XENCB_BF16: return run(read_attn_kernel<__nv_bfloat16>);
    default: return run(read_attn_kernel<float>);
  }
}

size_t xencb_read_forced_workspace(int n_chunks, int d_s) {
  if (n_chunks <= 0 || d_s <= 0) return 0;
  return 2 * align_up((size_t)n_chunks * d_s * sizeof(float), 256);
}

int xencb_read_forced(const float* fa, int d_s, const void* slots, const void* vslots, int slots_dtype,
                      int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                      const int32_t* n_valid, int n_chunks, const float* r0, int64_t n_rows, int norm_match,
                      float* r_out, float* scale_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!fa || !slots || !page_of || !n_valid || !r_out)
    return fail(XENCB_EINVAL, "read_forced: fa, slots, page_of, n_valid and r_out are required");
  if (d_s <= 0 || page_rows <= 0 || n_chunks <= 0 || n_rows <= 0 || n_pages <= 0)
    return fail(XENCB_EINVAL, "read_forced: sizes must be positive");
  if (norm_match && !r0) return fail(XENCB_EINVAL, "read_forced: force_norm_match needs r0 (the ordinary read)");
  const int es = elem_size(slots_dtype);
  if (!es) return fail(XENCB_EINVAL, "read_forced: slots_dtype %d unknown", slots_dtype);
  if (page_stride < (int64_t)page_rows * d_s)
    return fail(XENCB_EINVAL, "read_forced: page_stride %lld < page_rows*d_s", (long long)page_stride);
  const size_t one = align_up((size_t)n_chunks * d_s * sizeof(float), 256);
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < 2 * one)
    return fail(XENCB_EINVAL, "read_forced: workspace needs %zu bytes, 256-byte aligned (got %zu)", 2 * one,
                workspace_bytes);
  float* part_v = static_cast<float*>(workspace);
  float* part_k = reinterpret_cast<float*>(static_cast<char*>(workspace) + one);
  const bool untied = vslots != nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)n_chunks, (unsigned)((d_s + 4 * AT_THREADS - 1) / (4 * AT_THREADS)));
  auto run = [&](auto kern) -> int {
    kern<<<grid, AT_THREADS, 0, st>>>(fa, d_s, static_cast<const char*>(untied ? vslots : slots), n_pages,
                                      page_stride * es, page_rows, page_of, n_valid, part_v);
    XENCB_CHECK_LAUNCH("forced_partial launch");
    if (untied && norm_match) {  // the norm is taken on K (xenc/injector.py:252-254), the read on V
      kern<<<grid, AT_THREADS, 0, st>>>(fa, d_s, static_cast<const char*>(slots), n_pages, page_stride * es,
                                        page_rows, page_of, n_valid, part_k);
      XENCB_CHECK_LAUNCH("forced_partial launch");
    }
    forced_rows_kernel<<<(unsigned)n_rows, AT_THREADS, 0, st>>>(part_v, (untied && norm_match) ? part_k : part_v,
                                                               n_chunks, d_s, norm_match ? r0 : nullptr, r_out,
                                                               scale_out);
    XENCB_CHECK_LAUNCH("forced_rows launch");
    return XENCB_OK;
  };
  switch (slots_dtype) {
    case XENCB_F16: return run(forced_partial_kernel<__half>);
    case XENCB_BF16: return run(forced_partial_kernel<__nv_bfloat16>);
    default: return run(forced_partial_kernel<float>);
  }
}

int xencb_read_decode_noalloc(const float* q, int64_t n_rows, int d_s, const void* slots, int slots_dtype,
                              int64_t n_pages, int64_t page_stride, int page_rows, const int32_t* page_of,
                              const int32_t* n_valid, int n_chunks, int64_t rows_per_lib, int64_t n_lib,
                              const int32_t* idx, const float* wk, int k, float read_temp, int read_softmax,
                              float* r_out, void* stream) {
  const size_t need = (n_rows > 0 && k > 0 && d_s > 0 && page_rows > 0)
                          ? xencb_read_decode_workspace(n_rows, k, d_s, page_rows, slots_dtype)
                          : 0;
  if (need > (size_t)XENCB_NOALLOC_SCRATCH_BYTES)
    return fail(XENCB_EINVAL,
                "read_decode_noalloc: this call needs %zu bytes of scratch, more than the library's fixed "
                "%zu-byte device array; use xencb_read_decode with a caller workspace, or fewer rows per call",
                need, (size_t)XENCB_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
  }
  // need == 0 means invalid arguments: xencb_read_decode reports which one (it checks them before the workspace)
  return xencb_read_decode(q, n_rows, d_s, slots, nullptr, slots_dtype, n_pages, page_stride, page_rows, page_of, n_valid,
                           n_chunks, rows_per_lib, n_lib, idx, wk, k, read_temp, read_softmax, r_out, scratch,
                           need > 0 ? (size_t)XENCB_NOALLOC_SCRATCH_BYTES : 0, stream);
}

}  // extern "C"

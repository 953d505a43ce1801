// Projection GEMM, fp32-faithful on the f16 tensor cores ("3xF16"), tcgen05 + TMEM + TMA, split-K.
//
//   part[z][m][n] = sum_{k in split z} X[m][k] * W[n][k]         W: [N, K] (nn.Linear layout), X: [M, K]
//
// f16 carries the same 10 explicit mantissa bits as tf32, so splitting an fp32 value v into f16 hi = rn(v) and
// lo = rn(v - hi) keeps ~22 bits, and hi*hi + hi*lo + lo*hi (the dropped lo*lo is below 2^-22 relative) gives the
// accuracy of the 3xTF32 product, with twice the K per tensor-core instruction of kind::tf32 and half the
// operand bytes. f16 has a small exponent range, so both sides are scaled by powers of two first (exact):
//   * W once per weight tensor (xencb_weights_prep): s_w = 2^e with max|W| s_w in [2^14, 2^15), stored as f16
//     tiles of W_hi and W_lo (the same 4 bytes per weight as fp32; layout at split_weights_kernel) and 1 / s_w;
//   * X per call and per row (split_rows_f16x2_kernel): s_m = 2^e_m from the row's max |x|, rows stacked
//     [X_hi; X_lo] ([2M, K]) with 1 / s_m per row.
// Values far below a row's (or the weight's) maximum lose relative precision in f16's subnormal range; their
// share of a dot product is below 2^-28 of its largest term.
//
// gemm_f16x3_kernel: D[n][m] = W[n, :] . X[m, :] (128 output features = UMMA M, up to 64 tokens = UMMA N).
// Warp 0 lane 0 TMA-loads per 64-column k-block the tile pair W_hi, W_lo [2 x 128 x 64] (one contiguous 32 KiB
// run of the prepared weight, so a CTA's k-blocks are one sequential stream) and the boxes X_hi, X_lo [64 x 64],
// all 128-byte-swizzled, into a 4- or 2-stage ring (weights with L2 evict-last); warp 1 lane 0 issues 4 k-steps
// x 3 tcgen05.mma kind::f16 (f32 accumulate in TMEM) per k-block and commits each stage back to the producer;
// warps 2-5 read the accumulator (tcgen05.ld), undo the scales and store the split partial. Weight rows past N
// and columns past K are zeros in the prepared tiles; X boxes that run past M read rows of the other half of
// the stacked pair or zeros, which only reach outputs m >= M (not stored). Every barrier wait is bounded; TMEM
// is freed on every path.
#pragma once

#include "tc.cuh"

namespace xencb {

constexpr int H3_BM = 128;  // output features per CTA (UMMA M)
constexpr int H3_BN = 64;   // tokens per CTA (UMMA N)
constexpr int H3_BK = 64;   // K per k-block: 64 f16 = one 128-byte swizzle row
constexpr int H3_WBOX = H3_BM * H3_BK * 2;  // 16 KiB
constexpr int H3_XBOX = H3_BN * H3_BK * 2;  // 8 KiB
constexpr int H3_STAGE = 2 * H3_WBOX + 2 * H3_XBOX;  // W_hi | W_lo | X_hi | X_lo
constexpr int H3_THREADS = 32 * 6;
// Two shapes of the kernel: one CTA per SM with a 4-stage ring when all rows fit one 64-row tile (decode: the
// split-K CTAs each stream a short run of k-blocks), two CTAs per SM with 2 stages each for more rows (prefill:
// one CTA's prologue and epilogue overlap the other's stream; measured 3.6 % faster at config 3, and 1.6 %
// slower at config 2).
__host__ __device__ constexpr size_t h3_smem(int stages) { return 1024 + (size_t)stages * H3_STAGE + 256; }
constexpr uint32_t H3_TMEM_COLS = 64;
constexpr int WPREP_HEAD = 256;  // bytes before the tiles of a prepared weight: float max_bits, float inv_scale
constexpr int WPREP_PAIR = 2 * H3_BM * H3_BK;  // halves per tile pair (W_hi tile, then W_lo tile): 32 KiB

// Tile pairs of a prepared [n, k] weight: 128-row bands x 64-column blocks.
__host__ __device__ inline int64_t wprep_pairs(int64_t n, int64_t k) {
  return ((n + H3_BM - 1) / H3_BM) * ((k + H3_BK - 1) / H3_BK);
}

// 2^e with max * 2^e in [2^14, 2^15) (e = 0 for max 0 or non-finite): exact power-of-two scale into f16 range.
__device__ __forceinline__ float f16_range_scale(float mx) {
  if (!(mx > 0.f) || !isfinite(mx)) return 1.f;
  int ex;
  frexpf(mx, &ex);  // mx = f * 2^ex, f in [0.5, 1)
  return ldexpf(1.f, 15 - ex);
}

template <typename T>
__device__ __forceinline__ void split_f16(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

// Weight prep, pass 1: max |W| into the head's first word (float bits compare as unsigned for x >= 0).
__global__ void __launch_bounds__(256) absmax_kernel(const float* __restrict__ w, int64_t n, unsigned int* out) {
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(w[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// Weight prep, pass 2: the tiles of W_hi and W_lo with the scale from pass 1, and 1 / s_w into the head.
// Layout: tile pair p = band * KB + block (KB = ceil(k / 64) blocks per band; band = 128 rows of W, block = 64
// columns) at p * 32 KiB: the band's 128 x 64 f16 tile of W_hi, then the one of W_lo, each row-major (128 bytes
// a row). Rows past n and columns past k are zeros. Each thread writes 8 consecutive halves of a tile row
// (k % 8 == 0, so a group of 8 is either all inside k or all past it).
__global__ void __launch_bounds__(256) split_weights_kernel(const float* __restrict__ w, int n, int k,
                                                            const unsigned int* __restrict__ maxbits,
                                                            __half* __restrict__ tiles,
                                                            float* __restrict__ inv_scale) {
  const float s = f16_range_scale(__uint_as_float(*maxbits));
  if (blockIdx.x == 0 && threadIdx.x == 0) *inv_scale = 1.f / s;
  const int KB = (k + H3_BK - 1) / H3_BK;
  const int64_t groups = wprep_pairs(n, k) * (H3_BM * H3_BK / 8);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = g / (H3_BM * H3_BK / 8);
    const int r = (int)(g / (H3_BK / 8)) % H3_BM, c8 = (int)(g % (H3_BK / 8));
    const int row = (int)(p / KB) * H3_BM + r, col = (int)(p % KB) * H3_BK + c8 * 8;
    const bool in = row < n && col < k;  // scalar loads: w needs no more than float alignment
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = in ? w[(int64_t)row * k + col + e] : 0.f;
    alignas(16) __half h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) split_f16<float>(v[e] * s, h[e], l[e]);
    __half* dst = tiles + p * WPREP_PAIR + r * H3_BK + c8 * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(dst + H3_BM * H3_BK) = *reinterpret_cast<const uint4*>(l);
  }
}

// X per call: one CTA per row, [X_hi; X_lo] rows scaled by the row's own power of two, 1 / s_m per row. The row
// is read in 8-element pieces kept in registers between the max and the split (K <= 8 * 256 * SR_PIECES).
constexpr int SR_THREADS = 256;
constexpr int SR_PIECES = 4;

template <typename T>
__device__ __forceinline__ void load8_f32(const T* p, float* v) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    unpack16<T>(*reinterpret_cast<const uint4*>(p), v);
  }
}

template <typename T>
__global__ void __launch_bounds__(SR_THREADS) split_rows_f16x2_kernel(const T* __restrict__ x, int64_t M, int K,
                                                                      __half* __restrict__ hi, __half* __restrict__ lo,
                                                                      float* __restrict__ inv_scale) {
  __shared__ float red[SR_THREADS / 32];
  pdl_trigger();  // the GEMM that follows may start on its weight tiles now
  pdl_wait();
  const int64_t m = blockIdx.x;
  const T* xr = x + m * K;
  float v[SR_PIECES][8];
  float mx = 0.f;
#pragma unroll
  for (int p = 0; p < SR_PIECES; ++p) {
    const int k = (p * SR_THREADS + threadIdx.x) * 8;
    if (k < K) {
      load8_f32<T>(xr + k, v[p]);
#pragma unroll
      for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[p][e]));
    }
  }
  // pieces beyond SR_PIECES (rows longer than 8 * 256 * SR_PIECES): the max over a second read
  for (int k = (SR_PIECES * SR_THREADS + threadIdx.x) * 8; k < K; k += SR_THREADS * 8) {
    float w[8];
    load8_f32<T>(xr + k, w);
#pragma unroll
    for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(w[e]));
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  float rm = 0.f;
#pragma unroll
  for (int w = 0; w < SR_THREADS / 32; ++w) rm = fmaxf(rm, red[w]);
  const float s = f16_range_scale(rm);
  if (threadIdx.x == 0) inv_scale[m] = 1.f / s;
  auto emit = [&](int k, const float* w) {
    alignas(16) __half h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) split_f16<float>(w[e] * s, h[e], l[e]);
    *reinterpret_cast<uint4*>(hi + m * K + k) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(lo + m * K + k) = *reinterpret_cast<const uint4*>(l);
  };
#pragma unroll
  for (int p = 0; p < SR_PIECES; ++p) {
    const int k = (p * SR_THREADS + threadIdx.x) * 8;
    if (k < K) emit(k, v[p]);
  }
  for (int k = (SR_PIECES * SR_THREADS + threadIdx.x) * 8; k < K; k += SR_THREADS * 8) {
    float w[8];
    load8_f32<T>(xr + k, w);
    emit(k, w);
  }
}

template <int STAGES, int MINB>
__global__ void __launch_bounds__(H3_THREADS, MINB) gemm_f16x3_kernel(const __grid_constant__ CUtensorMap map_w,
                                                                   const __grid_constant__ CUtensorMap map_x,
                                                                   int64_t M, int N, int K, int kps,
                                                                   const float* __restrict__ w_inv_scale,
                                                                   const float* __restrict__ x_inv_scale,
                                                                   float* __restrict__ part, int* __restrict__ row_done) {
  extern __shared__ unsigned char h3_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(h3_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * H3_STAGE);
  uint64_t* sfree = full + STAGES;
  uint64_t* done = sfree + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * H3_BM;
  const int64_t m0 = (int64_t)blockIdx.y * H3_BN;
  const int kbeg = blockIdx.z * kps;
  const int kend = min(K, kbeg + kps);
  const int nkb = kend > kbeg ? (kend - kbeg + H3_BK - 1) / H3_BK : 0;
  // the prepared weight's tile-pair rows: pair (band blockIdx.x, block kb) starts at row 256 * pair
  const int wrow0 = (blockIdx.x * ((K + H3_BK - 1) / H3_BK) + kbeg / H3_BK) * 2 * H3_BM;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_w);
    prefetch_tensormap(&map_x);
  }
  if (warp == 1) {
    tc_alloc(tmem_slot, H3_TMEM_COLS);
    tc_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sfree[i], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;
  // Under programmatic dependent launch the producer requests the weight tiles of the first stage before the
  // row split this GEMM reads has finished (no kernel of the step writes the weights); everything else waits.
  // One stage, not the whole ring: measured in the decode steps, requesting every stage early competes with the
  // kernels still running (config 2: 162.3 -> 161.2 us per step, config 4: 607 -> 597 us with one stage).
  const int npre = min(nkb, 1);
  if (threadIdx.x != 0) {
    pdl_wait();
    pdl_trigger();
  }
  // zero the per-row completion counters the following reduce kernel counts on (stream order)
  if (row_done && blockIdx.x == 0 && blockIdx.z == 0)
    for (int64_t i = m0 + threadIdx.x; i < min(M, m0 + H3_BN); i += blockDim.x)
      if (threadIdx.x != 0) row_done[i] = 0;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      for (int kb = 0; kb < npre; ++kb) {
        unsigned char* st = smem + kb * H3_STAGE;
        mbar_arrive_expect_tx(&full[kb], H3_STAGE);
        tma_load_2d_hint(st, &map_w, 0, wrow0 + kb * 2 * H3_BM, &full[kb], keep);
      }
      pdl_wait();
      pdl_trigger();
      if (row_done && blockIdx.x == 0 && blockIdx.z == 0 && m0 < M) row_done[m0] = 0;
      for (int kb = 0; kb < npre; ++kb) {
        unsigned char* st = smem + kb * H3_STAGE;
        const int k = kbeg + kb * H3_BK;
        tma_load_2d(st + 2 * H3_WBOX, &map_x, k, (int)m0, &full[kb]);
        tma_load_2d(st + 2 * H3_WBOX + H3_XBOX, &map_x, k, (int)(M + m0), &full[kb]);
      }
      for (int kb = npre; kb < nkb; ++kb) {
        const int s = kb % STAGES, use = kb / STAGES;
        if (use > 0 && (!mbar_wait_spin(&sfree[s], (use - 1) & 1) || *abort_flag)) { *abort_flag = 1; break; }
        unsigned char* st = smem + s * H3_STAGE;
        mbar_arrive_expect_tx(&full[s], H3_STAGE);
        const int k = kbeg + kb * H3_BK;
        tma_load_2d_hint(st, &map_w, 0, wrow0 + kb * 2 * H3_BM, &full[s], keep);  // W_hi then W_lo tile
        tma_load_2d(st + 2 * H3_WBOX, &map_x, k, (int)m0, &full[s]);
        tma_load_2d(st + 2 * H3_WBOX + H3_XBOX, &map_x, k, (int)(M + m0), &full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(UMMA_F16, UMMA_F16, H3_BM, H3_BN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait_spin(&full[s], (kb / STAGES) & 1) || *abort_flag) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t sb = smem_u32(smem + s * H3_STAGE);
        const uint32_t wh = sb, wl = sb + H3_WBOX, xh = sb + 2 * H3_WBOX, xl = xh + H3_XBOX;
#pragma unroll
        for (int ks = 0; ks < H3_BK / 16; ++ks) {  // 16 f16 per UMMA k-step: 32 bytes along the swizzle row
          const uint32_t off = ks * 32;
          tc_mma<0>(taddr, umma_desc_k_sw128(wh + off), umma_desc_k_sw128(xh + off), idesc, kb > 0 || ks > 0);
          tc_mma<0>(taddr, umma_desc_k_sw128(wh + off), umma_desc_k_sw128(xl + off), idesc, true);
          tc_mma<0>(taddr, umma_desc_k_sw128(wl + off), umma_desc_k_sw128(xh + off), idesc, true);
        }
        tc_commit(&sfree[s]);  // the stage is free once these MMAs have read it
      }
      tc_commit(done);
    }
  } else {
    // ------------------------------------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int n = n0 + q * 32 + lane;
    float* out = part + (int64_t)blockIdx.z * M * N;
    // the scales are read while the MMAs run: one row scale per lane (rows m0 + lane, m0 + 32 + lane), handed to
    // the other lanes by shuffles; only the accumulator columns that hold rows are read back
    const float iw = *w_inv_scale;
    const float xs0 = m0 + lane < M ? x_inv_scale[m0 + lane] : 0.f;
    const float xs1 = m0 + 32 + lane < M ? x_inv_scale[m0 + 32 + lane] : 0.f;
    const int rows = (int)min((int64_t)H3_BN, M - m0);
    const bool ok = nkb > 0 && mbar_wait_bounded(done, 0) && !*abort_flag;
    tc_fence_after();
    for (int c = 0; c < rows; c += 32) {
      float v[32];
      tc_ld32(taddr + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
      const float xs = c == 0 ? xs0 : xs1;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float sm = __shfl_sync(0xffffffffu, xs, i);
        if (c + i < rows && n < N) out[(m0 + c + i) * N + n] = ok ? v[i] * iw * sm : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tc_dealloc(taddr, H3_TMEM_COLS);
}

}  // namespace xencb

// Projection GEMM on the 5th-generation tensor cores: 3xTF32 (fp32-faithful) split-K, tcgen05 + TMEM + TMA.
//
//   part[z][m][n] = sum_{k in split z} X[m][k] * W[n][k]         W: [N, K] (torch nn.Linear layout), X: [M, K]
//
// The product is computed transposed, D[n][m] = W[n, :] . X[m, :], so the 128 output features of a CTA are the
// UMMA M dimension and up to 64 tokens its N dimension (decode batches are small). Per 32-wide k-block:
//   * warp 0 / lane 0 TMA-loads the W tile [128 x 32] and the X tile [64 x 32] (fp32, 128-byte swizzle);
//   * warps 2-5 split both tiles in place into a tf32 "hi" part (low 13 mantissa bits cleared) and write the
//     exact remainder "lo" = x - hi beside them, then fence the async proxy;
//   * warp 1 / lane 0 issues 4 k-steps x 3 tcgen05.mma (hi*hi + hi*lo + lo*hi, kind::tf32, f32 accumulate in
//     TMEM) and commits to the stage's "empty" barrier, releasing it to the producer.
// After the last k-block the same four warps read the 128 x 64 accumulator out of TMEM (tcgen05.ld, one lane
// quarter each) and store the split partial. The dropped lo*lo term and the tf32 truncation of lo leave a
// relative error near 2^-21 per product.
// Every barrier wait is bounded; TMEM (64 columns) is freed on every path.
#pragma once

#include "tc.cuh"

namespace xencb {

constexpr int TC_BM = 128;  // output features per CTA (UMMA M)
constexpr int TC_BN = 64;   // tokens per CTA (UMMA N)
constexpr int TC_BK = 32;   // fp32 per 128-byte swizzle row = one k-block
constexpr int TC_STAGES = 4;
constexpr int TC_W_BYTES = TC_BM * TC_BK * 4;                  // 16 KiB
constexpr int TC_X_BYTES = TC_BN * TC_BK * 4;                  // 8 KiB
constexpr int TC_STAGE_BYTES = 2 * TC_W_BYTES + 2 * TC_X_BYTES;  // W, W_lo, X, X_lo
constexpr int TC_THREADS = 192;
constexpr size_t TC_SMEM = 1024 + (size_t)TC_STAGES * TC_STAGE_BYTES + 256;
constexpr uint32_t TC_TMEM_COLS = 64;

__device__ __forceinline__ void tf32_split4(float4& x, float4& lo) {
  const uint32_t m = 0xFFFFE000u;
  float h;
  h = __uint_as_float(__float_as_uint(x.x) & m); lo.x = x.x - h; x.x = h;
  h = __uint_as_float(__float_as_uint(x.y) & m); lo.y = x.y - h; x.y = h;
  h = __uint_as_float(__float_as_uint(x.z) & m); lo.z = x.z - h; x.z = h;
  h = __uint_as_float(__float_as_uint(x.w) & m); lo.w = x.w - h; x.w = h;
}

__global__ void __launch_bounds__(TC_THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w,
                                                                const __grid_constant__ CUtensorMap map_x,
                                                                int64_t M, int N, int K, int kps,
                                                                float* __restrict__ part, int* __restrict__ row_done) {
  extern __shared__ unsigned char tc_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE_BYTES);
  uint64_t* ready = full + TC_STAGES;
  uint64_t* empty = ready + TC_STAGES;
  uint64_t* done = empty + TC_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TC_BM;
  const int64_t m0 = (int64_t)blockIdx.y * TC_BN;
  const int kbeg = blockIdx.z * kps;
  const int kend = min(K, kbeg + kps);
  const int nkb = kend > kbeg ? (kend - kbeg + TC_BK - 1) / TC_BK : 0;

  // zero the per-row completion counters the following reduce kernel counts on (stream order)
  if (row_done && blockIdx.x == 0 && blockIdx.z == 0)
    for (int64_t i = m0 + threadIdx.x; i < min(M, m0 + TC_BN); i += blockDim.x) row_done[i] = 0;
  if (warp == 1) {
    tc_alloc(tmem_slot, TC_TMEM_COLS);
    tc_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&ready[i], 4);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------- producer
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % TC_STAGES, use = kb / TC_STAGES;
        if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1)) { *abort_flag = 1; break; }
        unsigned char* st = smem + s * TC_STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], TC_W_BYTES + TC_X_BYTES);
        const int k = kbeg + kb * TC_BK;
        tma_load_2d(st, &map_w, k, n0, &full[s]);
        tma_load_2d(st + 2 * TC_W_BYTES, &map_x, k, (int)m0, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(UMMA_TF32, UMMA_TF32, TC_BM, TC_BN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % TC_STAGES, use = kb / TC_STAGES;
        if (!mbar_wait_bounded(&ready[s], use & 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * TC_STAGE_BYTES);
        const uint32_t w_hi = st, w_lo = st + TC_W_BYTES, x_hi = st + 2 * TC_W_BYTES, x_lo = x_hi + TC_X_BYTES;
#pragma unroll
        for (int ks = 0; ks < TC_BK / 8; ++ks) {  // 8 tf32 = 32 bytes per UMMA k-step
          const uint32_t off = ks * 32;
          tc_mma<1>(taddr, umma_desc_k_sw128(w_hi + off), umma_desc_k_sw128(x_hi + off), idesc, kb > 0 || ks > 0);
          tc_mma<1>(taddr, umma_desc_k_sw128(w_hi + off), umma_desc_k_sw128(x_lo + off), idesc, true);
          tc_mma<1>(taddr, umma_desc_k_sw128(w_lo + off), umma_desc_k_sw128(x_hi + off), idesc, true);
        }
        tc_commit(&empty[s]);  // stage s is free once these MMAs have read it
      }
      tc_commit(done);
    }
  } else {
    // ------------------------------------------------------------------------------------------- split + epilogue
    const int ct = threadIdx.x - 64;  // 0..127
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % TC_STAGES, use = kb / TC_STAGES;
      if (!mbar_wait_bounded(&full[s], use & 1) || *abort_flag) { *abort_flag = 1; break; }
      unsigned char* st = smem + s * TC_STAGE_BYTES;
      float4* w = reinterpret_cast<float4*>(st);
      float4* wl = reinterpret_cast<float4*>(st + TC_W_BYTES);
      float4* x = reinterpret_cast<float4*>(st + 2 * TC_W_BYTES);
      float4* xl = reinterpret_cast<float4*>(st + 2 * TC_W_BYTES + TC_X_BYTES);
#pragma unroll
      for (int j = 0; j < TC_W_BYTES / 16 / 128; ++j) {  // the swizzle permutes 16-byte chunks: an
        const int i = ct + j * 128;                      // element-wise split keeps every position
        float4 v = w[i], lo;
        tf32_split4(v, lo);
        w[i] = v;
        wl[i] = lo;
      }
#pragma unroll
      for (int j = 0; j < TC_X_BYTES / 16 / 128; ++j) {
        const int i = ct + j * 128;
        float4 v = x[i], lo;
        tf32_split4(v, lo);
        x[i] = v;
        xl[i] = lo;
      }
      fence_proxy_async_smem();  // generic-proxy writes become visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[s]);
    }
    // epilogue: lane quarter (warp % 4) of the 128 x 64 accumulator
    const int q = warp & 3;
    const int n = n0 + q * 32 + lane;
    float* out = part + (int64_t)blockIdx.z * M * N;
    const bool ok = nkb > 0 && mbar_wait_bounded(done, 0) && !*abort_flag;
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < TC_BN; c += 16) {
      float v[16];
      tc_ld16(taddr + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t m = m0 + c + i;
        if (m < M && n < N) out[m * N + n] = ok ? v[i] : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tc_dealloc(taddr, TC_TMEM_COLS);
}

}  // namespace xencb

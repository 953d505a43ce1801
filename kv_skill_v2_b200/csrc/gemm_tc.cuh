// Projection GEMM on the 5th-generation tensor cores: 3xTF32 (fp32-faithful) split-K, tcgen05 + TMEM + TMA.
//
//   part[z][m][n] = sum_{k in split z} X[m][k] * W[n][k]         W: [N, K] (torch nn.Linear layout), X: [M, K]
//
// The product is computed transposed, D[n][m] = W[n, :] . X[m, :], so the 128 output features of a CTA are the
// UMMA M dimension and up to 64 tokens its N dimension (decode batches are small). A k-block is 64 columns of K,
// loaded as two 128-byte-swizzled boxes per operand:
//   * warp 0 / lane 0 TMA-loads the W boxes [128 x 32] x 2 (L2 evict_last: the weights are re-read every step)
//     and the X boxes [64 x 32] x 2 (fp32) into a landing stage;
//   * warps 2-9 split, one thread per (W row, box): split warp j (= warp - 2) takes box j / 4 and the rows of
//     TMEM lane quarter warp % 4 (the quarter a warp may access). A thread reads its row's 32 floats, splits them into a tf32 "hi" part (low 13 mantissa bits
//     cleared) and the exact remainder "lo" = x - hi, and writes both straight into tensor memory (tcgen05.st):
//     the A operand of the MMA lives in TMEM, so W costs no shared-memory bandwidth after the landing stage.
//     The X boxes are split the same way into a shared-memory operand buffer (the B operand). The landing stage
//     is free as soon as it has been read into registers;
//   * warp 1 / lane 0 issues 8 k-steps x 3 tcgen05.mma (hi*hi + hi*lo + lo*hi, kind::tf32, A from TMEM, f32
//     accumulate in TMEM) and commits to the operand buffer's "free" barrier.
// After the last k-block warps 2-5 read the 128 x 64 accumulator out of TMEM (tcgen05.ld, one lane quarter each)
// and store the split partial. The dropped lo*lo term and the tf32 truncation of lo leave a relative error near
// 2^-21 per product.
// TMEM (512 columns): accumulator [0, 64); operand buffer o: W_hi [64 + 128o, 128 + 128o), W_lo [128 + 128o,
// 192 + 128o). Every barrier wait is bounded; TMEM is freed on every path.
#pragma once

#include "tc.cuh"

namespace xencb {

constexpr int TC_BM = 128;  // output features per CTA (UMMA M)
constexpr int TC_BN = 64;   // tokens per CTA (UMMA N)
constexpr int TC_BOX = 32;  // fp32 per 128-byte swizzle row = one TMA box along K
constexpr int TC_BK = 2 * TC_BOX;  // K per k-block
constexpr int TC_TSTAGES = 3;  // TMA landing stages (W, X)
constexpr int TC_OBUFS = 2;    // operand buffers (W_hi, W_lo in TMEM; X_hi, X_lo in shared memory)
constexpr int TC_WBOX_BYTES = TC_BM * TC_BOX * 4;  // 16 KiB
constexpr int TC_XBOX_BYTES = TC_BN * TC_BOX * 4;  // 8 KiB
constexpr int TC_TSTAGE_BYTES = 2 * TC_WBOX_BYTES + 2 * TC_XBOX_BYTES;  // W box 0, W box 1, X box 0, X box 1
constexpr int TC_OBUF_BYTES = 4 * TC_XBOX_BYTES;                        // X_hi box 0, 1, X_lo box 0, 1
constexpr int TC_SPLIT_WARPS = 8;
constexpr int TC_THREADS = 32 * (2 + TC_SPLIT_WARPS);
constexpr size_t TC_SMEM = 1024 + (size_t)TC_TSTAGES * TC_TSTAGE_BYTES + (size_t)TC_OBUFS * TC_OBUF_BYTES + 256;
constexpr uint32_t TC_TMEM_COLS = 512;  // accumulator 64 + 2 operand buffers x (hi 64 + lo 64)
constexpr uint32_t TC_TMEM_A0 = 64;

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
  unsigned char* tstage = smem;                                        // [TC_TSTAGES][W0 | W1 | X0 | X1]
  unsigned char* obuf = smem + TC_TSTAGES * TC_TSTAGE_BYTES;           // [TC_OBUFS][Xh0 | Xh1 | Xl0 | Xl1]
  uint64_t* full = reinterpret_cast<uint64_t*>(obuf + TC_OBUFS * TC_OBUF_BYTES);
  uint64_t* tfree = full + TC_TSTAGES;
  uint64_t* ready = tfree + TC_TSTAGES;
  uint64_t* ofree = ready + TC_OBUFS;
  uint64_t* done = ofree + TC_OBUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TC_BM;
  const int64_t m0 = (int64_t)blockIdx.y * TC_BN;
  const int kbeg = blockIdx.z * kps;
  const int kend = min(K, kbeg + kps);
  const int nkb = kend > kbeg ? (kend - kbeg + TC_BK - 1) / TC_BK : 0;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_w);
    prefetch_tensormap(&map_x);
  }
  // zero the per-row completion counters the following reduce kernel counts on (stream order)
  if (row_done && blockIdx.x == 0 && blockIdx.z == 0)
    for (int64_t i = m0 + threadIdx.x; i < min(M, m0 + TC_BN); i += blockDim.x) row_done[i] = 0;
  if (warp == 1) {
    tc_alloc(tmem_slot, TC_TMEM_COLS);
    tc_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_TSTAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&tfree[i], TC_SPLIT_WARPS);
    }
    for (int i = 0; i < TC_OBUFS; ++i) {
      mbar_init(&ready[i], TC_SPLIT_WARPS);
      mbar_init(&ofree[i], 1);
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
      const uint64_t keep = policy_evict_last();
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % TC_TSTAGES, use = kb / TC_TSTAGES;
        if (use > 0 && (!mbar_wait_bounded(&tfree[s], (use - 1) & 1) || *abort_flag)) { *abort_flag = 1; break; }
        unsigned char* st = tstage + s * TC_TSTAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], TC_TSTAGE_BYTES);
        const int k = kbeg + kb * TC_BK;
        tma_load_2d_hint(st, &map_w, k, n0, &full[s], keep);
        tma_load_2d_hint(st + TC_WBOX_BYTES, &map_w, k + TC_BOX, n0, &full[s], keep);
        tma_load_2d(st + 2 * TC_WBOX_BYTES, &map_x, k, (int)m0, &full[s]);
        tma_load_2d(st + 2 * TC_WBOX_BYTES + TC_XBOX_BYTES, &map_x, k + TC_BOX, (int)m0, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(UMMA_TF32, UMMA_TF32, TC_BM, TC_BN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int o = kb % TC_OBUFS, use = kb / TC_OBUFS;
        if (!mbar_wait_bounded(&ready[o], use & 1) || *abort_flag) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t ob = smem_u32(obuf + o * TC_OBUF_BYTES);
        const uint32_t a_hi = taddr + TC_TMEM_A0 + 128u * (uint32_t)o, a_lo = a_hi + 64u;
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          const uint32_t x_hi = ob + bx * TC_XBOX_BYTES, x_lo = ob + (2 + bx) * TC_XBOX_BYTES;
#pragma unroll
          for (int ks = 0; ks < TC_BOX / 8; ++ks) {  // 8 tf32 per UMMA k-step: 8 TMEM columns of A, 32 B of B
            const uint32_t off = ks * 32, acol = 32u * bx + 8u * ks;
            tc_mma_tf32_at(taddr, a_hi + acol, umma_desc_k_sw128(x_hi + off), idesc, kb > 0 || bx > 0 || ks > 0);
            tc_mma_tf32_at(taddr, a_hi + acol, umma_desc_k_sw128(x_lo + off), idesc, true);
            tc_mma_tf32_at(taddr, a_lo + acol, umma_desc_k_sw128(x_hi + off), idesc, true);
          }
        }
        tc_commit(&ofree[o]);  // the operand buffer is free once these MMAs have read it
      }
      tc_commit(done);
    }
  } else {
    // ------------------------------------------------------------------------------------------- split + epilogue
    const int sw = warp - 2;           // 0..7
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int bx = sw >> 2;            // the box (K columns [32 bx, 32 bx + 32)) this warp splits
    const int r = q * 32 + lane;       // its W row
    const int xt = (sw & 3) * 32 + lane;  // 0..127: its share of the box's X tile
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % TC_TSTAGES, o = kb % TC_OBUFS;
      if (!mbar_wait_bounded(&full[s], (kb / TC_TSTAGES) & 1) || *abort_flag) { *abort_flag = 1; break; }
      if (kb >= TC_OBUFS && (!mbar_wait_bounded(&ofree[o], ((kb / TC_OBUFS) - 1) & 1) || *abort_flag)) {
        *abort_flag = 1;
        break;
      }
      const unsigned char* st = tstage + s * TC_TSTAGE_BYTES;
      const float4* w = reinterpret_cast<const float4*>(st + bx * TC_WBOX_BYTES);
      const float4* x = reinterpret_cast<const float4*>(st + 2 * TC_WBOX_BYTES + bx * TC_XBOX_BYTES);
      unsigned char* ob = obuf + o * TC_OBUF_BYTES;
      float4* xh = reinterpret_cast<float4*>(ob + bx * TC_XBOX_BYTES);
      float4* xl = reinterpret_cast<float4*>(ob + (2 + bx) * TC_XBOX_BYTES);
      // this thread's W row (128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8))
      float hi[TC_BOX], lo[TC_BOX];
#pragma unroll
      for (int c = 0; c < TC_BOX / 4; ++c) {
        const float4 v = w[r * (TC_BOX / 4) + (c ^ (r & 7))];
        hi[4 * c] = v.x; hi[4 * c + 1] = v.y; hi[4 * c + 2] = v.z; hi[4 * c + 3] = v.w;
      }
      float4 vx[TC_XBOX_BYTES / 16 / 128];
#pragma unroll
      for (int j = 0; j < TC_XBOX_BYTES / 16 / 128; ++j) vx[j] = x[xt + j * 128];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[s]);  // the landing stage has been read into registers
#pragma unroll
      for (int i = 0; i < TC_BOX; ++i) {
        const float h = __uint_as_float(__float_as_uint(hi[i]) & 0xFFFFE000u);
        lo[i] = hi[i] - h;
        hi[i] = h;
      }
      const uint32_t ta = taddr + ((uint32_t)(q * 32) << 16) + TC_TMEM_A0 + 128u * (uint32_t)o + 32u * (uint32_t)bx;
      tc_st32(ta, hi);
      tc_st32(ta + 64u, lo);
      // the X box: element-wise split at the same (swizzled) offsets
#pragma unroll
      for (int j = 0; j < TC_XBOX_BYTES / 16 / 128; ++j) {
        float4 l4;
        tf32_split4(vx[j], l4);
        xh[xt + j * 128] = vx[j];
        xl[xt + j * 128] = l4;
      }
      tc_wait_st();
      fence_proxy_async_smem();  // generic-proxy writes become visible to the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[o]);
    }
    // epilogue (warps 2-5): lane quarter q of the 128 x 64 accumulator
    if (sw < 4) {
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
    } else if (nkb > 0) {
      mbar_wait_bounded(done, 0);  // every MMA has finished before TMEM is released below
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tc_dealloc(taddr, TC_TMEM_COLS);
}

}  // namespace xencb

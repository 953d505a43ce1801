// Interface projections at both ends of the read (float32 arithmetic, as the reference's read_fp32 path).
//
//   project_in : q = L2(rms_norm(h) @ W_in^T + b), gate = sigmoid(hn . gate_w + gate_b), selector logits
//   project_out: delta = scale * gate * (r @ W_out^T + b) -> selector matched norm -> position mask ->
//                cast to h's dtype -> mag term and h + delta
//
// The contraction runs as a split-K SIMT GEMM (Y_part[z] = X[:, Kz] @ W[:, Kz]^T) into a caller-provided
// workspace; a per-row "finish" kernel then reduces the splits and applies every elementwise step, so the
// full output row is available for the L2 / matched-norm reductions. rms_norm's 1/rms factor is applied to
// the GEMM result (it is a per-row scalar), which keeps h in its storage type on the GEMM's input side.
#pragma once

#include "common.cuh"

namespace xencb {

constexpr int GEMM_BM = 64, GEMM_BN = 128, GEMM_BK = 16, GEMM_THREADS = 128;
constexpr int GEMM_APAD = GEMM_BM + 4, GEMM_BPAD = GEMM_BN + 4;

// part[z][m][n] = sum_{k in [z*kps, min(K,(z+1)*kps))} X[m][k] * W[n][k]
// grid: (ceil(N/BN), ceil(M/BM), splits); block 128 threads, each an 8x8 register tile.
template <typename TX>
__global__ void __launch_bounds__(GEMM_THREADS) gemm_tn_splitk_kernel(const TX* __restrict__ X, int64_t M, int K,
                                                                       const float* __restrict__ W, int N, int kps,
                                                                       float* __restrict__ part) {
  __shared__ __align__(16) float As[2][GEMM_BK][GEMM_APAD];
  __shared__ __align__(16) float Bs[2][GEMM_BK][GEMM_BPAD];

  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;  // 8 x 16 thread grid
  const int64_t m0 = (int64_t)blockIdx.y * GEMM_BM;
  const int n0 = blockIdx.x * GEMM_BN;
  const int kbeg = blockIdx.z * kps;
  const int kend = min(K, kbeg + kps);

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  // staging registers: A tile 64x16 = 1024 elems -> 8 per thread; B tile 128x16 = 2048 -> 16 per thread
  float ra[8], rb[16];
  auto load_tile = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int f = tid + i * GEMM_THREADS;  // 0..1023
      const int mm = f >> 4, kk = f & 15;
      const int64_t gm = m0 + mm;
      const int gk = k0 + kk;
      ra[i] = (gm < M && gk < kend) ? to_f32(X[gm * K + gk]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int f = tid + i * GEMM_THREADS;  // 0..2047
      const int nn = f >> 4, kk = f & 15;
      const int gn = n0 + nn;
      const int gk = k0 + kk;
      rb[i] = (gn < N && gk < kend) ? __ldg(W + (int64_t)gn * K + gk) : 0.f;
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int f = tid + i * GEMM_THREADS;
      As[buf][f & 15][f >> 4] = ra[i];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int f = tid + i * GEMM_THREADS;
      Bs[buf][f & 15][f >> 4] = rb[i];
    }
  };

  if (kbeg < kend) {
    load_tile(kbeg);
    store_tile(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = kbeg; k0 < kend; k0 += GEMM_BK) {
      const bool more = k0 + GEMM_BK < kend;
      if (more) load_tile(k0 + GEMM_BK);
#pragma unroll
      for (int kk = 0; kk < GEMM_BK; ++kk) {
        const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8]);
        const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8 + 4]);
        const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
        const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
        const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      if (more) {
        store_tile(buf ^ 1);
        __syncthreads();
        buf ^= 1;
      }
    }
  }

  float* out = part + (int64_t)blockIdx.z * M * N;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + ty * 8 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn < N) out[gm * N + gn] = acc[i][j];
    }
  }
}

// Split count so that the GEMM grid covers the SMs about twice; each split is a multiple of BK.
inline int gemm_splits(int64_t M, int N, int K, int sms) {
  const int64_t tiles = ((N + GEMM_BN - 1) / GEMM_BN) * ((M + GEMM_BM - 1) / GEMM_BM);
  const int kblocks = (K + GEMM_BK - 1) / GEMM_BK;
  int64_t s = (2 * (int64_t)sms + tiles - 1) / tiles;
  if (s < 1) s = 1;
  if (s > kblocks) s = kblocks;
  if (s > 32) s = 32;
  return (int)s;
}

inline int gemm_kps(int K, int splits) {
  const int kblocks = (K + GEMM_BK - 1) / GEMM_BK;
  return ((kblocks + splits - 1) / splits) * GEMM_BK;
}

// ------------------------------------------------------------------------------------------------ project_in
// One CTA per row: 1/rms of h, reduce the GEMM splits, bias, L2, gate, selector logits.
template <typename TH>
__global__ void __launch_bounds__(256) project_in_finish_kernel(
    const TH* __restrict__ h, int d_m, const float* __restrict__ part, int splits, int64_t M, int d_s, int flags,
    const float* __restrict__ b_in, const float* __restrict__ gate_w, float gate_b,
    const float* __restrict__ sel_w, const float* __restrict__ sel_b, int n_cand, float eps,
    float* __restrict__ q_out, float* __restrict__ gate_out, float* __restrict__ rstd_out,
    float* __restrict__ z_out) {
  __shared__ float red[32];
  __shared__ float zsh[32];
  const int64_t row = blockIdx.x;
  const TH* hr = h + row * d_m;

  // rms_norm scale
  float ss = 0.f, gd = 0.f;
  for (int i = threadIdx.x; i < d_m; i += blockDim.x) {
    const float x = to_f32(hr[i]);
    ss = fmaf(x, x, ss);
    if (gate_w) gd = fmaf(x, gate_w[i], gd);
  }
  ss = block_sum(ss, red);
  const float rstd = (flags & XENCB_PIN_RMS) ? rsqrtf(ss / (float)d_m + eps) : 1.f;
  if (gate_w) {
    gd = block_sum(gd, red);
    if (threadIdx.x == 0) {
      const float zg = gd * rstd + gate_b;
      gate_out[row] = 1.f / (1.f + expf(-zg));
    }
  }
  if (rstd_out && threadIdx.x == 0) rstd_out[row] = rstd;

  // selector logits: one warp per candidate
  if (sel_w) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int c = wid; c < n_cand; c += nw) {
      const float* u = sel_w + (int64_t)c * d_m;
      float d = 0.f;
      for (int i = lane; i < d_m; i += 32) d = fmaf(to_f32(hr[i]), u[i], d);
      d = warp_sum(d);
      if (lane == 0) zsh[c] = d * rstd + (sel_b ? sel_b[c] : 0.f);
    }
    __syncthreads();
    if (threadIdx.x < n_cand) z_out[row * n_cand + threadIdx.x] = zsh[threadIdx.x];
  }

  // q = rstd * sum_z part + b, then L2
  float* qr = q_out + row * d_s;
  float nq = 0.f;
  for (int n = threadIdx.x; n < d_s; n += blockDim.x) {
    float v = 0.f;
    for (int z = 0; z < splits; ++z) v += part[((int64_t)z * M + row) * d_s + n];
    v = v * rstd + (b_in ? b_in[n] : 0.f);
    qr[n] = v;
    nq = fmaf(v, v, nq);
  }
  if (flags & XENCB_PIN_L2) {
    nq = block_sum(nq, red);
    const float den = sqrtf(nq) + 1e-6f;
    for (int n = threadIdx.x; n < d_s; n += blockDim.x) qr[n] = qr[n] / den;
  }
}

// rms_norm rows: out = h * rsqrt(mean(h^2) + eps); one CTA per row.
template <typename TH>
__global__ void __launch_bounds__(256) rms_norm_kernel(const TH* __restrict__ h, int d_m, float eps,
                                                      float* __restrict__ out) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const TH* hr = h + row * d_m;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d_m; i += blockDim.x) { const float x = to_f32(hr[i]); ss = fmaf(x, x, ss); }
  ss = block_sum(ss, red);
  const float rstd = rsqrtf(ss / (float)d_m + eps);
  for (int i = threadIdx.x; i < d_m; i += blockDim.x) out[row * d_m + i] = to_f32(hr[i]) * rstd;
}

// ------------------------------------------------------------------------------------------------ project_out
// One CTA per row. Dynamic smem: d_m floats holding the row of delta in float32.
template <typename TH>
__global__ void __launch_bounds__(256) project_out_finish_kernel(
    const float* __restrict__ part, int splits, int64_t M, int d_m, const float* __restrict__ b_out, float scale,
    const float* __restrict__ gate, const float* __restrict__ sel_w, float alpha, const float* __restrict__ pos_mask,
    const TH* h, TH* delta_out, TH* h_out, float* __restrict__ rel_out) {
  extern __shared__ float drow[];
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float g = (gate ? gate[row] : 1.f) * scale;

  float dd = 0.f, hh = 0.f;
  for (int n = threadIdx.x; n < d_m; n += blockDim.x) {
    float v = 0.f;
    for (int z = 0; z < splits; ++z) v += part[((int64_t)z * M + row) * d_m + n];
    v = g * (v + (b_out ? b_out[n] : 0.f));
    drow[n] = v;
    dd = fmaf(v, v, dd);
    const float x = to_f32(h[row * d_m + n]);
    hh = fmaf(x, x, hh);
  }
  dd = block_sum(dd, red);
  hh = block_sum(hh, red);
  const float hnorm = sqrtf(hh);
  // LayerSelector.apply: d / (||d|| / (||h|| + eps) + eps) * exp(log_alpha), then * w[..., pos]
  const float rel_d = sqrtf(dd) / (hnorm + 1e-6f) + 1e-6f;
  const float sw = sel_w ? sel_w[row] : 1.f;
  const float pm = pos_mask ? pos_mask[row] : 1.f;

  float cn = 0.f;
  for (int n = threadIdx.x; n < d_m; n += blockDim.x) {
    float v = drow[n];
    if (sel_w) v = sw * ((v / rel_d) * alpha);
    if (pos_mask) v *= pm;
    const TH dv = from_f32<TH>(v);
    const float dvf = to_f32(dv);
    cn = fmaf(dvf, dvf, cn);
    if (delta_out) delta_out[row * d_m + n] = dv;
    if (h_out) h_out[row * d_m + n] = from_f32<TH>(to_f32(h[row * d_m + n]) + dvf);
  }
  if (rel_out) {
    cn = block_sum(cn, red);
    if (threadIdx.x == 0) rel_out[row] = sqrtf(cn) / (hnorm + 1e-6f);
  }
}

// LayerSelector.apply on a given delta: one CTA per row (norms of delta and h, then the rescale).
template <typename TD, typename TH>
__global__ void __launch_bounds__(256) selector_apply_kernel(const TD* delta, const TH* __restrict__ h, int d,
                                                            const float* __restrict__ w, int n_cand, int pos,
                                                            float alpha, TD* out) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  float dd = 0.f, hh = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float x = to_f32(delta[row * d + i]);
    const float y = to_f32(h[row * d + i]);
    dd = fmaf(x, x, dd);
    hh = fmaf(y, y, hh);
  }
  dd = block_sum(dd, red);
  hh = block_sum(hh, red);
  const float rel = sqrtf(dd) / (sqrtf(hh) + 1e-6f) + 1e-6f;
  const float wp = w[row * n_cand + pos];
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float x = to_f32(delta[row * d + i]);
    out[row * d + i] = from_f32<TD>(wp * ((x / rel) * alpha));
  }
}

}  // namespace xencb

// Interface projections at both ends of the read (float32 arithmetic, as the reference's read_fp32 path).
//
//   project_in : q = L2(rms_norm(h) @ W_in^T + b), gate = sigmoid(hn . gate_w + gate_b), selector logits
//   project_out: delta = scale * gate * (r @ W_out^T + b) -> selector matched norm -> position mask ->
//                cast to h's dtype -> mag term and h + delta
//
// The contraction runs as a split-K GEMM (Y_part[z] = X[:, Kz] @ W[:, Kz]^T, gemm_tc.cuh on the tensor cores, or the
// SIMT fallback below) into a caller-provided workspace; a per-row "finish" kernel then reduces the splits and applies every elementwise step, so the
// full output row is available for the L2 / matched-norm reductions. rms_norm's 1/rms factor is applied to
// the GEMM result (it is a per-row scalar), which keeps h in its storage type on the GEMM's input side.
#pragma once

#include "common.cuh"

namespace xencb {

// SIMT fallback GEMM (shapes the TMA path cannot take: K % 4 != 0 or unaligned rows), torch nn.Linear
// weight layout W [N, K]:
constexpr int SG_BM = 64, SG_BN = 128, SG_BK = 16, SG_THREADS = 128;
constexpr int SG_APAD = SG_BM + 4, SG_BPAD = SG_BN + 4;

// part[z][m][n] = sum_{k in [z*kps, min(K,(z+1)*kps))} X[m][k] * W[n][k]
// grid: (ceil(N/BN), ceil(M/BM), splits); block 128 threads, each an 8x8 register tile.
template <typename TX>
__global__ void __launch_bounds__(SG_THREADS) gemm_simt_splitk_kernel(const TX* __restrict__ X, int64_t M, int K,
                                                                       const float* __restrict__ W, int N, int kps,
                                                                       float* __restrict__ part,
                                                                       int* __restrict__ row_done) {
  if (row_done && blockIdx.x == 0 && blockIdx.z == 0)
    for (int64_t i = (int64_t)blockIdx.y * SG_BM + threadIdx.x; i < min(M, (int64_t)(blockIdx.y + 1) * SG_BM);
         i += blockDim.x)
      row_done[i] = 0;
  __shared__ __align__(16) float As[2][SG_BK][SG_APAD];
  __shared__ __align__(16) float Bs[2][SG_BK][SG_BPAD];

  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;  // 8 x 16 thread grid
  const int64_t m0 = (int64_t)blockIdx.y * SG_BM;
  const int n0 = blockIdx.x * SG_BN;
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
      const int f = tid + i * SG_THREADS;  // 0..1023
      const int mm = f >> 4, kk = f & 15;
      const int64_t gm = m0 + mm;
      const int gk = k0 + kk;
      ra[i] = (gm < M && gk < kend) ? to_f32(X[gm * K + gk]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int f = tid + i * SG_THREADS;  // 0..2047
      const int nn = f >> 4, kk = f & 15;
      const int gn = n0 + nn;
      const int gk = k0 + kk;
      rb[i] = (gn < N && gk < kend) ? __ldg(W + (int64_t)gn * K + gk) : 0.f;
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int f = tid + i * SG_THREADS;
      As[buf][f & 15][f >> 4] = ra[i];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int f = tid + i * SG_THREADS;
      Bs[buf][f & 15][f >> 4] = rb[i];
    }
  };

  if (kbeg < kend) {
    load_tile(kbeg);
    store_tile(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = kbeg; k0 < kend; k0 += SG_BK) {
      const bool more = k0 + SG_BK < kend;
      if (more) load_tile(k0 + SG_BK);
#pragma unroll
      for (int kk = 0; kk < SG_BK; ++kk) {
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
inline int sg_splits(int64_t M, int N, int K, int sms) {
  const int64_t tiles = ((N + SG_BN - 1) / SG_BN) * ((M + SG_BM - 1) / SG_BM);
  const int kblocks = (K + SG_BK - 1) / SG_BK;
  int64_t s = (2 * (int64_t)sms + tiles - 1) / tiles;
  if (s < 1) s = 1;
  if (s > kblocks) s = kblocks;
  if (s > 32) s = 32;
  return (int)s;
}

inline int sg_kps(int K, int splits) {
  const int kblocks = (K + SG_BK - 1) / SG_BK;
  return ((kblocks + splits - 1) / splits) * SG_BK;
}

// Sum of the split partials of 4 consecutive columns (col % 4 == 0, N % 4 == 0), loads kept independent.
__device__ __forceinline__ float4 sum_splits4(const float* __restrict__ part, int splits, int64_t M, int N,
                                              int64_t row, int col) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  const float* p = part + row * N + col;
  const int64_t zs = M * N;
  int z = 0;
  for (; z + 4 <= splits; z += 4) {
    float4 t[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) t[u] = *reinterpret_cast<const float4*>(p + (int64_t)(z + u) * zs);
#pragma unroll
    for (int u = 0; u < 4; ++u) { v.x += t[u].x; v.y += t[u].y; v.z += t[u].z; v.w += t[u].w; }
  }
  for (; z < splits; ++z) {
    const float4 t = *reinterpret_cast<const float4*>(p + (int64_t)z * zs);
    v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
  }
  return v;
}

// Split sums of VPT float4 column groups (columns n[v], v < VPT; ok[v] false for none) with 16 / VPT splits'
// loads of each in flight, added in split order: the same sums as sum_splits4.
template <int VPT>
__device__ __forceinline__ void sum_splits_row(const float* __restrict__ part, int splits, int64_t M, int N,
                                               int64_t row, const int* n, const bool* ok, float4* v) {
  constexpr int SB = 16 / VPT;
  const int64_t zs = M * N;
#pragma unroll
  for (int q = 0; q < VPT; ++q) v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int z0 = 0; z0 < splits; z0 += SB) {
    float4 t[VPT][SB];
#pragma unroll
    for (int q = 0; q < VPT; ++q)
#pragma unroll
      for (int u = 0; u < SB; ++u)
        if (ok[q] && z0 + u < splits)
          t[q][u] = *reinterpret_cast<const float4*>(part + row * N + n[q] + (int64_t)(z0 + u) * zs);
#pragma unroll
    for (int q = 0; q < VPT; ++q)
#pragma unroll
      for (int u = 0; u < SB; ++u)
        if (ok[q] && z0 + u < splits) {
          v[q].x += t[q][u].x; v[q].y += t[q][u].y; v[q].z += t[q][u].z; v[q].w += t[q][u].w;
        }
  }
}

// Two block-wide sums in one pass (blockDim.x <= 1024); `red2` holds 32 float2.
__device__ __forceinline__ float2 block_sum2(float a, float b, float2* red2) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  __syncthreads();
  if (lane == 0) red2[wid] = make_float2(a, b);
  __syncthreads();
  const float2 t = lane < nw ? red2[lane] : make_float2(0.f, 0.f);
  return make_float2(warp_sum(t.x), warp_sum(t.y));
}

// Row passes with 16-byte loads, four in flight per thread: sum of x^2, and sum of x*w for up to two vectors.
template <typename TH>
__device__ __forceinline__ void row_dots(const TH* __restrict__ hr, int d, const float* __restrict__ w1,
                                         const float* __restrict__ w2, float& ss, float& s1, float& s2) {
  constexpr int EPV = 16 / sizeof(TH);
  ss = s1 = s2 = 0.f;
  const bool vec = (d % EPV == 0) && ((reinterpret_cast<uintptr_t>(hr) & 15) == 0) &&
                   (!w1 || (reinterpret_cast<uintptr_t>(w1) & 15) == 0) &&
                   (!w2 || (reinterpret_cast<uintptr_t>(w2) & 15) == 0);
  if (vec) {
    const uint4* h4 = reinterpret_cast<const uint4*>(hr);
    const int nv = d / EPV;
#pragma unroll 4
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
      float x[EPV];
      unpack16<TH>(__ldg(h4 + v), x);
#pragma unroll
      for (int e = 0; e < EPV; ++e) {
        ss = fmaf(x[e], x[e], ss);
        if (w1) s1 = fmaf(x[e], __ldg(w1 + v * EPV + e), s1);
        if (w2) s2 = fmaf(x[e], __ldg(w2 + v * EPV + e), s2);
      }
    }
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
      const float x = to_f32(hr[i]);
      ss = fmaf(x, x, ss);
      if (w1) s1 = fmaf(x, w1[i], s1);
      if (w2) s2 = fmaf(x, w2[i], s2);
    }
  }
}

// ------------------------------------------------------------------------------------------------ project_in
// Two launches after the GEMM. project_in_reduce: one CTA per (row, 1024-column chunk) sums the split
// partials (independent 16-byte loads), applies 1/rms and the bias, writes the unnormalised row and the
// chunk's sum of squares; the chunk-0 CTA also writes 1/rms, the gate and the selector logits.
// project_in_normalize: one CTA per row divides by ||q|| + 1e-6 (the reference's L2, xenc/injector.py:58).
constexpr int PIN_CHUNK = 1024;  // columns per reduce CTA (256 threads x 4)

template <typename TH>
__global__ void __launch_bounds__(256) project_in_reduce_kernel(
    const TH* __restrict__ h, int d_m, const float* __restrict__ part, int splits, int64_t M, int d_s, int flags,
    const float* __restrict__ b_in, const float* __restrict__ gate_w, float gate_b, const float* __restrict__ gate_b_dev,
    const float* __restrict__ sel_w, const float* __restrict__ sel_b, int n_cand, float eps,
    float* __restrict__ q_out, float* __restrict__ nq_part, int* __restrict__ row_done, float* __restrict__ gate_out,
    float* __restrict__ rstd_out, float* __restrict__ z_out) {
  __shared__ float red[32];
  __shared__ float zsh[32];
  const int64_t row = blockIdx.x;
  const int chunk = blockIdx.y;
  const TH* hr = h + row * d_m;

  float ss, gd, unused;
  row_dots<TH>(hr, d_m, chunk == 0 ? gate_w : nullptr, nullptr, ss, gd, unused);
  float rstd = 1.f;
  if (flags & XENCB_PIN_RMS) {  // every chunk CTA needs 1/rms; the row is 4-16 KB and L2-resident
    ss = block_sum(ss, red);
    rstd = rsqrtf(ss / (float)d_m + eps);
  }
  if (chunk == 0) {
    if (rstd_out && threadIdx.x == 0) rstd_out[row] = (flags & XENCB_PIN_RMS) ? rstd : 1.f;
    if (gate_w) {
      gd = block_sum(gd, red);
      const float gb = gate_b_dev ? __ldg(gate_b_dev) : gate_b;
      if (threadIdx.x == 0) gate_out[row] = 1.f / (1.f + expf(-(gd * rstd + gb)));
    }
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
  }
  float nq = 0.f;
  const int n = chunk * PIN_CHUNK + threadIdx.x * 4;
  if (n < d_s) {
    const float4 v = sum_splits4(part, splits, M, d_s, row, n);
    float4 o;
    o.x = v.x * rstd + (b_in ? b_in[n] : 0.f);
    o.y = v.y * rstd + (b_in ? b_in[n + 1] : 0.f);
    o.z = v.z * rstd + (b_in ? b_in[n + 2] : 0.f);
    o.w = v.w * rstd + (b_in ? b_in[n + 3] : 0.f);
    *reinterpret_cast<float4*>(q_out + row * d_s + n) = o;
    nq = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
  }
  __threadfence();  // this CTA's q columns are visible to whichever CTA normalises the row
  nq = block_sum(nq, red);
  if (!(flags & XENCB_PIN_L2)) return;
  // the CTA that finishes a row last divides the whole row by ||q|| + 1e-6 (chunk sums in a fixed order)
  __shared__ int last;
  if (threadIdx.x == 0) {
    nq_part[row * gridDim.y + chunk] = nq;
    __threadfence();
    last = atomicAdd(&row_done[row], 1) == (int)gridDim.y - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float tot = 0.f;
  for (int c = 0; c < (int)gridDim.y; ++c) tot += __ldcg(nq_part + row * gridDim.y + c);
  const float den = sqrtf(tot) + 1e-6f;
  float* qr = q_out + row * d_s;
  for (int m = threadIdx.x * 4; m < d_s; m += blockDim.x * 4) {
    float4 o = __ldcg(reinterpret_cast<const float4*>(qr + m));
    o.x /= den; o.y /= den; o.z /= den; o.w /= den;
    *reinterpret_cast<float4*>(qr + m) = o;
  }
}

// project_in after the GEMM in one launch when a row fits one CTA (d_s <= 4 * ROW_THREADS * VPT): thread t owns
// the float4 column groups t + v * blockDim.x. The pass over h (sum of squares, gate dot, the selector's logit
// dots) runs before the wait for the GEMM: this kernel starts only after the GEMM passed its own wait, so the row
// split that read h, and the kernel that wrote it, have completed; nothing is written before the wait. Then the
// split partials; one two-value block sum gives 1/rms and the gate; q = (sum of splits) * rstd + b stays in
// registers for the L2 norm (||q|| + 1e-6, xenc/injector.py:58), so nothing is written twice.
// The two halves are shared with the fused decode router (route.cuh), which continues from q in registers.
constexpr int ROW_THREADS = 512;

struct PinArgs {
  int d_m;
  const float* part;
  int splits;
  int64_t M;
  int d_s, flags;
  const float* b_in;
  const float* gate_w;
  float gate_b;
  const float* gate_b_dev;
  const float* sel_w;
  const float* sel_b;
  int n_cand;
  float eps;
  float* q_out;
  float* gate_out;
  float* rstd_out;
  float* z_out;
};

// First half (before the wait): (sum of h^2, gate dot); the selector's logit dots go to zsh[n_cand] (skipped when
// `sel` is false: a CTA that writes no outputs).
template <typename TH>
__device__ __forceinline__ float2 pin_row_pre(const TH* __restrict__ hr, const PinArgs& a, float* zsh,
                                              bool sel = true) {
  float ss, gd, unused;
  row_dots<TH>(hr, a.d_m, a.gate_w, nullptr, ss, gd, unused);
  if (a.sel_w && sel) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int c = wid; c < a.n_cand; c += nw) {
      const float* u = a.sel_w + (int64_t)c * a.d_m;
      float d = 0.f;
      for (int i = lane; i < a.d_m; i += 32) d = fmaf(to_f32(hr[i]), u[i], d);
      d = warp_sum(d);
      if (lane == 0) zsh[c] = d;
    }
  }
  return make_float2(ss, gd);
}

// Second half (after the wait): q's columns n[v] (ok[v]: inside d_s) in o[v], written to q_out; 1/rms, the gate
// and the selector logits written too (each output skipped when its pointer is null, all of them when `write` is
// false).
template <int VPT>
__device__ __forceinline__ void pin_row_post(const PinArgs& a, int64_t row, float2 pre, const float* zsh,
                                             float2* red2, float* red, float4* o, int* n, bool* ok,
                                             bool write = true) {
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    n[q] = (threadIdx.x + q * blockDim.x) * 4;
    ok[q] = n[q] < a.d_s;
  }
  float4 v[VPT];
  sum_splits_row<VPT>(a.part, a.splits, a.M, a.d_s, row, n, ok, v);
  const float2 t = block_sum2(pre.x, pre.y, red2);  // (its barrier also publishes zsh)
  const float rstd = (a.flags & XENCB_PIN_RMS) ? rsqrtf(t.x / (float)a.d_m + a.eps) : 1.f;
  if (write && threadIdx.x == 0) {
    if (a.rstd_out) a.rstd_out[row] = rstd;
    if (a.gate_w && a.gate_out) {
      const float gb = a.gate_b_dev ? __ldg(a.gate_b_dev) : a.gate_b;
      a.gate_out[row] = 1.f / (1.f + expf(-(t.y * rstd + gb)));
    }
  }
  if (write && a.sel_w && a.z_out && threadIdx.x < a.n_cand)
    a.z_out[row * a.n_cand + threadIdx.x] = zsh[threadIdx.x] * rstd + (a.sel_b ? a.sel_b[threadIdx.x] : 0.f);
  float nq = 0.f;
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    o[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok[q]) {
      const int c = n[q];
      o[q].x = v[q].x * rstd + (a.b_in ? a.b_in[c] : 0.f);
      o[q].y = v[q].y * rstd + (a.b_in ? a.b_in[c + 1] : 0.f);
      o[q].z = v[q].z * rstd + (a.b_in ? a.b_in[c + 2] : 0.f);
      o[q].w = v[q].w * rstd + (a.b_in ? a.b_in[c + 3] : 0.f);
      nq += o[q].x * o[q].x + o[q].y * o[q].y + o[q].z * o[q].z + o[q].w * o[q].w;
    }
  }
  if (a.flags & XENCB_PIN_L2) {
    nq = block_sum(nq, red);
    const float den = sqrtf(nq) + 1e-6f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) { o[q].x /= den; o[q].y /= den; o[q].z /= den; o[q].w /= den; }
  }
  if (write && a.q_out) {
#pragma unroll
    for (int q = 0; q < VPT; ++q)
      if (ok[q]) *reinterpret_cast<float4*>(a.q_out + row * a.d_s + n[q]) = o[q];
  }
}

template <typename TH, int VPT>
__global__ void __launch_bounds__(ROW_THREADS) project_in_row_kernel(const TH* __restrict__ h, const PinArgs a) {
  __shared__ float2 red2[32];
  __shared__ float red[32];
  __shared__ float zsh[32];
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const float2 pre = pin_row_pre<TH>(h + row * a.d_m, a, zsh);
  pdl_wait();
  float4 o[VPT];
  int n[VPT];
  bool ok[VPT];
  pin_row_post<VPT>(a, row, pre, zsh, red2, red, o, n, ok);
}

// X as float32 rows for the TMA path (hidden states stored in 16-bit types).
template <typename TH>
__global__ void __launch_bounds__(256) to_f32_kernel(const TH* __restrict__ x, int64_t n, float* __restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = to_f32(x[i]);
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
// project_out_reduce: one CTA per (row, 1024-column chunk): d = scale * gate * (sum of split partials + bias)
// into the workspace, plus the chunk's sums of d^2 and h^2. project_out_epilogue: one CTA per row: the
// selector's matched norm, the position mask, the cast to h's dtype, h + delta and the mag term.
template <typename TH>
__global__ void __launch_bounds__(256) project_out_reduce_kernel(
    const float* __restrict__ part, int splits, int64_t M, int d_m, const float* __restrict__ b_out, float scale,
    const float* __restrict__ log_scale_dev, const float* __restrict__ gate, const TH* __restrict__ h,
    float* __restrict__ d_out,
    float* __restrict__ norm_part, int* __restrict__ row_done) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int chunk = blockIdx.y;
  if (chunk == 0 && threadIdx.x == 0) row_done[row] = 0;  // the epilogue's per-row counter
  const float g = (gate ? gate[row] : 1.f) * scale * (log_scale_dev ? expf(__ldg(log_scale_dev)) : 1.f);
  float dd = 0.f, hh = 0.f;
  const int n = chunk * PIN_CHUNK + threadIdx.x * 4;
  if (n < d_m) {
    const float4 v = sum_splits4(part, splits, M, d_m, row, n);
    float4 o;
    o.x = g * (v.x + (b_out ? b_out[n] : 0.f));
    o.y = g * (v.y + (b_out ? b_out[n + 1] : 0.f));
    o.z = g * (v.z + (b_out ? b_out[n + 2] : 0.f));
    o.w = g * (v.w + (b_out ? b_out[n + 3] : 0.f));
    *reinterpret_cast<float4*>(d_out + row * d_m + n) = o;
    dd = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
#pragma unroll
    for (int u = 0; u < 4; ++u) { const float y = to_f32(h[row * d_m + n + u]); hh = fmaf(y, y, hh); }
  }
  dd = block_sum(dd, red);
  hh = block_sum(hh, red);
  if (threadIdx.x == 0) {
    norm_part[(row * gridDim.y + chunk) * 2] = dd;
    norm_part[(row * gridDim.y + chunk) * 2 + 1] = hh;
  }
}

template <typename TH>
__global__ void __launch_bounds__(256) project_out_epilogue_kernel(
    const float* __restrict__ d_in, const float* __restrict__ norm_part, int d_m, const float* __restrict__ sel_w,
    float alpha_host, const float* __restrict__ log_alpha_dev, const float* __restrict__ pos_mask, const TH* h, TH* delta_out, TH* h_out, float* __restrict__ rel_out,
    float* __restrict__ cn_part, int* __restrict__ row_done) {
  __shared__ float red[32];
  __shared__ int last;
  const int64_t row = blockIdx.x;
  const int chunk = blockIdx.y, n_chunks = gridDim.y;
  float dd = 0.f, hh = 0.f;
  for (int c = 0; c < n_chunks; ++c) {
    dd += norm_part[(row * n_chunks + c) * 2];
    hh += norm_part[(row * n_chunks + c) * 2 + 1];
  }
  const float hnorm = sqrtf(hh);
  // LayerSelector.apply: d / (||d|| / (||h|| + eps) + eps) * exp(log_alpha), then * w[..., pos]
  const float rel_d = sqrtf(dd) / (hnorm + 1e-6f) + 1e-6f;
  const float sw = sel_w ? sel_w[row] : 1.f;
  const float pm = pos_mask ? pos_mask[row] : 1.f;
  const float alpha = log_alpha_dev ? expf(__ldg(log_alpha_dev)) : alpha_host;
  float cn = 0.f;
  const int n = chunk * PIN_CHUNK + threadIdx.x * 4;
  if (n < d_m) {
    const float4 v4 = *reinterpret_cast<const float4*>(d_in + row * d_m + n);
    const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float v = vv[u];
      if (sel_w) v = sw * ((v / rel_d) * alpha);
      if (pos_mask) v *= pm;
      const TH dv = from_f32<TH>(v);
      const float dvf = to_f32(dv);
      cn = fmaf(dvf, dvf, cn);
      if (delta_out) delta_out[row * d_m + n + u] = dv;
      if (h_out) h_out[row * d_m + n + u] = from_f32<TH>(to_f32(h[row * d_m + n + u]) + dvf);
    }
  }
  if (!rel_out) return;
  cn = block_sum(cn, red);
  // the CTA that finishes a row last sums the chunk norms in a fixed order
  if (threadIdx.x == 0) {
    cn_part[row * n_chunks + chunk] = cn;
    __threadfence();
    last = atomicAdd(&row_done[row], 1) == n_chunks - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    float tot = 0.f;
    for (int c = 0; c < n_chunks; ++c) tot += __ldcg(cn_part + row * n_chunks + c);
    rel_out[row] = sqrtf(tot) / (hnorm + 1e-6f);
  }
}

// project_out after the GEMM in one launch when a row fits one CTA (d_m <= 4 * ROW_THREADS * VPT): thread t owns
// the float4 column groups t + v * blockDim.x. d = scale * gate * (sum of splits + bias) stays in registers; one
// two-value block sum gives ||d|| and ||h||, then the epilogue of project_out_epilogue_kernel (the selector's
// matched norm, the position mask, the cast to h's dtype, h + delta) and, when asked, the block sum of the cast
// delta's squares for the mag term. h_out may alias h: every thread reads its own columns of h before the block
// sum and writes them after.
template <typename TH, int VPT>
__global__ void __launch_bounds__(ROW_THREADS) project_out_row_kernel(
    const float* __restrict__ part, int splits, int64_t M, int d_m, const float* __restrict__ b_out, float scale,
    const float* __restrict__ log_scale_dev, const float* __restrict__ gate, const TH* h,
    const float* __restrict__ sel_w, float alpha_host, const float* __restrict__ log_alpha_dev,
    const float* __restrict__ pos_mask, TH* delta_out, TH* h_out, float* __restrict__ rel_out) {
  __shared__ float2 red2[32];
  __shared__ float red[32];
  // h is the hook's input, complete before the step's first kernel: its row is read (and ||h|| summed) before the
  // wait; the next kernel may start its own early work now. Nothing is written before the wait.
  pdl_trigger();
  const int64_t row = blockIdx.x;
  int n[VPT];
  bool ok[VPT];
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    n[q] = (threadIdx.x + q * blockDim.x) * 4;
    ok[q] = n[q] < d_m;
  }
  float hx[VPT][4];
  float hh = 0.f;
#pragma unroll
  for (int q = 0; q < VPT; ++q)
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      hx[q][u] = ok[q] ? to_f32(h[row * d_m + n[q] + u]) : 0.f;
      hh = fmaf(hx[q][u], hx[q][u], hh);
    }
  pdl_wait();
  float4 v[VPT];
  sum_splits_row<VPT>(part, splits, M, d_m, row, n, ok, v);
  const float g = (gate ? gate[row] : 1.f) * scale * (log_scale_dev ? expf(__ldg(log_scale_dev)) : 1.f);
  float o[VPT][4];
  float dd = 0.f;
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    const int c = n[q];
    o[q][0] = ok[q] ? g * (v[q].x + (b_out ? b_out[c] : 0.f)) : 0.f;
    o[q][1] = ok[q] ? g * (v[q].y + (b_out ? b_out[c + 1] : 0.f)) : 0.f;
    o[q][2] = ok[q] ? g * (v[q].z + (b_out ? b_out[c + 2] : 0.f)) : 0.f;
    o[q][3] = ok[q] ? g * (v[q].w + (b_out ? b_out[c + 3] : 0.f)) : 0.f;
    dd += o[q][0] * o[q][0] + o[q][1] * o[q][1] + o[q][2] * o[q][2] + o[q][3] * o[q][3];
  }
  const float2 t = block_sum2(dd, hh, red2);
  const float hnorm = sqrtf(t.y);
  // LayerSelector.apply: d / (||d|| / (||h|| + eps) + eps) * exp(log_alpha), then * w[..., pos]
  const float rel_d = sqrtf(t.x) / (hnorm + 1e-6f) + 1e-6f;
  const float sw = sel_w ? sel_w[row] : 1.f;
  const float pm = pos_mask ? pos_mask[row] : 1.f;
  const float alpha = log_alpha_dev ? expf(__ldg(log_alpha_dev)) : alpha_host;
  float cn = 0.f;
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    if (!ok[q]) continue;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x = o[q][u];
      if (sel_w) x = sw * ((x / rel_d) * alpha);
      if (pos_mask) x *= pm;
      const TH dv = from_f32<TH>(x);
      const float dvf = to_f32(dv);
      cn = fmaf(dvf, dvf, cn);
      if (delta_out) delta_out[row * d_m + n[q] + u] = dv;
      if (h_out) h_out[row * d_m + n[q] + u] = from_f32<TH>(hx[q][u] + dvf);
    }
  }
  if (!rel_out) return;
  cn = block_sum(cn, red);
  if (threadIdx.x == 0) rel_out[row] = sqrtf(cn) / (hnorm + 1e-6f);
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

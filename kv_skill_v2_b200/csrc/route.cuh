// Chunk routing (xenc/injector.py:220-229), LayerSelector weights (xenc/selector.py:59-67) and the
// Library's summary keys (xenc/library.py:69-74).
//
// Routing: the logits q . S * route_temp (the reference's order: dot first, then the temperature), then per row k
// rounds of a warp arg-max with ties to the lower chunk index and the softmax over the kept logits. Decode (few
// rows per Library) runs both in route_fused_kernel, an 8-CTA cluster per row gathering the logits in the
// leader's shared memory; prefill-sized batches run route_logits_tiled_kernel, then route_topk_kernel.
#pragma once

#include <math_constants.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "project.cuh"

namespace xencb {

namespace cg = cooperative_groups;

// q . S over d_s fp32 columns for one warp (result in every lane); q is normally the caller's shared-memory copy
// of the row (read by every warp of the CTA), S streams from HBM. Lanes take 16-byte vectors i = lane + 32 j and
// accumulate j = 0, 4, 8, ... into d, j = 1, 5, ... into d1 and so on, combined as (d + d1) + (d2 + d3), then a
// xor-shuffle tree. The first loop keeps sixteen S vectors of a lane in flight (8 KB a warp: a d_s = 2048 row in
// one round trip); the second takes four at a time; both add in that same order, so the value does not depend on
// how many vectors were in flight.
__device__ __forceinline__ float route_dot(const float* qr, const float* __restrict__ sr, int d_s,
                                           int lane) {
  float d = 0.f;
  if ((d_s & 3) == 0) {
    const float4* q4 = reinterpret_cast<const float4*>(qr);
    const float4* s4 = reinterpret_cast<const float4*>(sr);
    const int n4 = d_s >> 2;
    float d1 = 0.f, d2 = 0.f, d3 = 0.f;
    int i = lane;
    for (; i + 480 < n4; i += 512) {
      float4 b[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) b[u] = __ldcs(s4 + i + 32 * u);
#pragma unroll
      for (int u = 0; u < 16; u += 4) {
        const float4 a0 = q4[i + 32 * u], a1 = q4[i + 32 * (u + 1)];
        const float4 a2 = q4[i + 32 * (u + 2)], a3 = q4[i + 32 * (u + 3)];
        d = fmaf(a0.x, b[u].x, d); d = fmaf(a0.y, b[u].y, d); d = fmaf(a0.z, b[u].z, d); d = fmaf(a0.w, b[u].w, d);
        d1 = fmaf(a1.x, b[u + 1].x, d1); d1 = fmaf(a1.y, b[u + 1].y, d1);
        d1 = fmaf(a1.z, b[u + 1].z, d1); d1 = fmaf(a1.w, b[u + 1].w, d1);
        d2 = fmaf(a2.x, b[u + 2].x, d2); d2 = fmaf(a2.y, b[u + 2].y, d2);
        d2 = fmaf(a2.z, b[u + 2].z, d2); d2 = fmaf(a2.w, b[u + 2].w, d2);
        d3 = fmaf(a3.x, b[u + 3].x, d3); d3 = fmaf(a3.y, b[u + 3].y, d3);
        d3 = fmaf(a3.z, b[u + 3].z, d3); d3 = fmaf(a3.w, b[u + 3].w, d3);
      }
    }
    for (; i + 96 < n4; i += 128) {
      const float4 b0 = __ldcs(s4 + i), b1 = __ldcs(s4 + i + 32), b2 = __ldcs(s4 + i + 64), b3 = __ldcs(s4 + i + 96);
      const float4 a0 = q4[i], a1 = q4[i + 32], a2 = q4[i + 64], a3 = q4[i + 96];
      d = fmaf(a0.x, b0.x, d); d = fmaf(a0.y, b0.y, d); d = fmaf(a0.z, b0.z, d); d = fmaf(a0.w, b0.w, d);
      d1 = fmaf(a1.x, b1.x, d1); d1 = fmaf(a1.y, b1.y, d1); d1 = fmaf(a1.z, b1.z, d1); d1 = fmaf(a1.w, b1.w, d1);
      d2 = fmaf(a2.x, b2.x, d2); d2 = fmaf(a2.y, b2.y, d2); d2 = fmaf(a2.z, b2.z, d2); d2 = fmaf(a2.w, b2.w, d2);
      d3 = fmaf(a3.x, b3.x, d3); d3 = fmaf(a3.y, b3.y, d3); d3 = fmaf(a3.z, b3.z, d3); d3 = fmaf(a3.w, b3.w, d3);
    }
    for (; i < n4; i += 32) {
      const float4 a = q4[i], b = __ldcs(s4 + i);
      d = fmaf(a.x, b.x, d); d = fmaf(a.y, b.y, d); d = fmaf(a.z, b.z, d); d = fmaf(a.w, b.w, d);
    }
    d = (d + d1) + (d2 + d3);
  } else {
    for (int i = lane; i < d_s; i += 32) d = fmaf(qr[i], __ldg(sr + i), d);
  }
  return warp_sum(d);
}

// Routing logits, few rows per Library: CTA (row, RL_CH-chunk block), 8 warps of RL_CH / 8 dot products each. The
// Ask L2 for a warp's first S row (lane l: 128-byte lines 2l and 2l+1 of up to 8 KB) before the CTA stages q,
// so the row is on its way while q is copied.
__device__ __forceinline__ void prefetch_row_l2(const float* sr, int d_s, int lane) {
  const char* p = reinterpret_cast<const char*>(sr);
  const int bytes = d_s * 4;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int off = (2 * lane + u) * 128;
    if (off < bytes) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + off));
  }
}

// row's q is staged in shared memory once (STAGE; dynamic smem d_s floats), else read from global memory.
constexpr int RL_CH = 16;
template <bool STAGE>
__global__ void __launch_bounds__(256) route_logits_kernel(const float* __restrict__ q, int64_t n_rows, int d_s,
                                                          const float* __restrict__ S, int C,
                                                          const int32_t* __restrict__ n_chunks_of,
                                                          int64_t rows_per_lib, float temp,
                                                          float* __restrict__ logit) {
  extern __shared__ float rl_q[];
  const int64_t row = blockIdx.x;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qr = q + row * d_s;
  const int64_t lib = row / rows_per_lib;
  const int c_first = blockIdx.y * RL_CH + w;
  if (c_first < C) prefetch_row_l2(S + (lib * C + c_first) * (int64_t)d_s, d_s, lane);
  if (STAGE) {
    for (int i = threadIdx.x; i < d_s; i += blockDim.x) rl_q[i] = qr[i];
    __syncthreads();
    qr = rl_q;
  }
  const int nc = n_chunks_of ? min(n_chunks_of[lib], C) : C;
  const int c_end = min(C, (int)(blockIdx.y + 1) * RL_CH);
  for (int c = blockIdx.y * RL_CH + w; c < c_end; c += 8) {
    if (c >= nc) {
      if (lane == 0) logit[row * C + c] = -CUDART_INF_F;
      continue;
    }
    const float d = route_dot(qr, S + (lib * C + c) * (int64_t)d_s, d_s, lane);
    if (lane == 0) logit[row * C + c] = d * temp;
  }
}

// Routing logits for many rows per Library (prefill): one CTA computes a 32-row x 64-chunk tile of
// logit = (q . S) * temp with both operands staged in shared memory in 32-column slices, so q and S are read
// once per tile instead of once per (row, chunk) dot. 256 threads, each 2 rows x 4 chunks in fp32 FMA.
constexpr int RT_ROWS = 32, RT_CH = 64, RT_K = 32;
__global__ void __launch_bounds__(256) route_logits_tiled_kernel(const float* __restrict__ q, int64_t n_rows, int d_s,
                                                                const float* __restrict__ S, int C,
                                                                const int32_t* __restrict__ n_chunks_of,
                                                                int64_t rows_per_lib, float temp,
                                                                float* __restrict__ logit) {
  __shared__ float qs[RT_ROWS][RT_K + 1];
  __shared__ float ss[RT_CH][RT_K + 1];
  const int64_t lib = blockIdx.z;
  const int64_t r0 = lib * rows_per_lib + (int64_t)blockIdx.x * RT_ROWS;  // first row of the tile
  int64_t r_lim = lib * rows_per_lib + rows_per_lib;
  if (r_lim > n_rows) r_lim = n_rows;
  const int c0 = blockIdx.y * RT_CH;
  const int nc = n_chunks_of ? min(n_chunks_of[lib], C) : C;
  const int tr = threadIdx.x >> 4;  // 0..15 -> rows tr, tr + 16
  const int tc = threadIdx.x & 15;  // 0..15 -> chunks tc + 16 j
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const float* Sl = S + lib * (int64_t)C * d_s;
  for (int k0 = 0; k0 < d_s; k0 += RT_K) {
    for (int i = threadIdx.x; i < RT_ROWS * RT_K; i += blockDim.x) {
      const int rr = i / RT_K, kk = i - rr * RT_K;
      const int64_t row = r0 + rr;
      qs[rr][kk] = (row < r_lim && k0 + kk < d_s) ? __ldg(q + row * d_s + k0 + kk) : 0.f;
    }
    for (int i = threadIdx.x; i < RT_CH * RT_K; i += blockDim.x) {
      const int cc = i / RT_K, kk = i - cc * RT_K;
      const int c = c0 + cc;
      ss[cc][kk] = (c < nc && k0 + kk < d_s) ? __ldg(Sl + (int64_t)c * d_s + k0 + kk) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < RT_K; ++kk) {
      const float a0 = qs[tr][kk], a1 = qs[tr + 16][kk];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float b = ss[tc + 16 * j][kk];
        acc[0][j] = fmaf(a0, b, acc[0][j]);
        acc[1][j] = fmaf(a1, b, acc[1][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t row = r0 + tr + 16 * i;
    if (row >= r_lim) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + tc + 16 * j;
      if (c < C) logit[row * C + c] = c < nc ? acc[i][j] * temp : -CUDART_INF_F;
    }
  }
}

// Warp arg-max over (value desc, index asc); returns the winner in every lane.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
}

constexpr int TOPK_WARPS = 4;

// topk_row for rows of up to 32 * TK_R chunks and k <= 32, with the logits held in registers (lane l owns chunks
// l + 32 i): each round is a register arg-max, a warp arg-max and a retire by the owning lane, with no shared
// memory and no warp barrier. Same selection, order and arithmetic as topk_row. lr may alias wd.
constexpr int TK_R = 8;
__device__ __forceinline__ void topk_row_reg(const float* lr, int C, int nc, int top_k, int k_out, float rw,
                                             int32_t* __restrict__ ir, float* __restrict__ wr, float* wd, int lane) {
  float x[TK_R];
#pragma unroll
  for (int i = 0; i < TK_R; ++i) {
    const int c = lane + 32 * i;
    x[i] = c < nc ? lr[c] : -CUDART_INF_F;
  }
  const bool skip = rw == 0.f;
  int mine = -1;
  float lmine = -CUDART_INF_F;
  for (int t = 0; t < top_k; ++t) {
    float bv = -CUDART_INF_F;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < TK_R; ++i) {
      const int c = lane + 32 * i;
      if (c < nc && (x[i] > bv || (x[i] == bv && c < bi))) { bv = x[i]; bi = c; }
    }
    warp_argmax(bv, bi);
    const int win = bi < nc ? bi : -1;  // -1 only with non-finite logits
    if (lane == t) { mine = win; lmine = bv; }
    if (win >= 0 && (win & 31) == lane) {
#pragma unroll
      for (int i = 0; i < TK_R; ++i)
        if (lane + 32 * i == win) x[i] = -CUDART_INF_F;
    }
  }
  const bool kept = lane < top_k && mine >= 0;
  if (!kept) lmine = -CUDART_INF_F;
  const float mx = warp_max(lmine);
  const float sum = warp_sum(kept ? expf(lmine - mx) : 0.f);
  const float wmine = kept ? expf(lmine - mx) / sum : 0.f;
  if (wd) {
    for (int c0 = 0; c0 < C; c0 += 32) {
      const int c = c0 + lane;
      float val = 0.f;
      for (int j = 0; j < top_k; ++j) {
        const int cj = __shfl_sync(0xffffffffu, mine, j);
        const float wj = __shfl_sync(0xffffffffu, wmine, j);
        if (cj == c) val = wj;
      }
      if (c < C) wd[c] = val;
    }
  }
  for (int j = lane; j < k_out; j += 32) {
    ir[j] = (skip || j >= top_k) ? -1 : mine;
    wr[j] = (skip || j >= top_k) ? 0.f : wmine;
  }
}

// Top-k and softmax of one row's logits lr[0, C) by one warp; v is the warp's scratch row of C floats (shared
// memory). Chunks at or past nc take no part. Sparse (0 < top_k < nc): top_k rounds of a warp arg-max (ties to
// the lower chunk), the winner retired to -inf in v, then the softmax over the kept logits. Dense: the softmax
// over all nc chunks, idx = 0..nc-1. A row whose weight rw is 0 reads nothing (idx -1); w_dense keeps its
// routing. lr may alias wd. Every output is written once, after all reads: a __syncwarp() after a global store
// orders that store, and waits for it, so no warp barrier follows one here.
__device__ __forceinline__ void topk_row(const float* lr, float* v, int C, int nc, int top_k, int k_out, float rw,
                                         int32_t* __restrict__ ir, float* __restrict__ wr, float* wd, int lane) {
  const bool sparse = top_k > 0 && top_k < nc;
  if (sparse && top_k <= 32 && C <= 32 * TK_R) {
    topk_row_reg(lr, C, nc, top_k, k_out, rw, ir, wr, wd, lane);
    return;
  }
  for (int c = lane; c < C; c += 32) v[c] = (c < nc) ? lr[c] : -CUDART_INF_F;
  __syncwarp();
  const bool skip = rw == 0.f;
  if (!sparse) {
    float mx = -CUDART_INF_F;
    for (int c = lane; c < nc; c += 32) mx = fmaxf(mx, v[c]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int c = lane; c < nc; c += 32) sum += expf(v[c] - mx);
    sum = warp_sum(sum);
    for (int j = lane; j < k_out; j += 32) {
      ir[j] = (j < nc && !skip) ? j : -1;
      wr[j] = (j < nc && !skip) ? expf(v[j] - mx) / sum : 0.f;
    }
    if (wd)
      for (int c = lane; c < C; c += 32) wd[c] = c < nc ? expf(v[c] - mx) / sum : 0.f;
    return;
  }
  // lane j keeps the winner of round j in a register; rounds 32 and up (k > 32, rare) go to ir
  int mine = -1;
  for (int t = 0; t < top_k; ++t) {
    float bv = -CUDART_INF_F;
    int bi = 0x7fffffff;
    for (int c = lane; c < nc; c += 32) {
      const float x = v[c];
      if (x > bv || (x == bv && c < bi)) { bv = x; bi = c; }
    }
    warp_argmax(bv, bi);
    const int win = bi < nc ? bi : -1;  // -1 only with non-finite logits
    if (t < 32) {
      if (lane == t) mine = win;
    } else if (lane == 0) {
      ir[t] = win;
    }
    if (lane == 0 && win >= 0) v[win] = -CUDART_INF_F;
    __syncwarp();
  }
  // softmax over the kept logits (the first one is the maximum); lr is read before anything is written to wd
  const bool kept = lane < top_k && mine >= 0;
  const float lmine = kept ? lr[mine] : -CUDART_INF_F;
  float mx = lmine;
  for (int j = 32 + lane; j < top_k; j += 32) { const int c = ir[j]; if (c >= 0) mx = fmaxf(mx, lr[c]); }
  mx = warp_max(mx);
  float sum = kept ? expf(lmine - mx) : 0.f;
  for (int j = 32 + lane; j < top_k; j += 32) { const int c = ir[j]; if (c >= 0) sum += expf(lr[c] - mx); }
  sum = warp_sum(sum);
  const float wmine = kept ? expf(lmine - mx) / sum : 0.f;
  for (int j = 32 + lane; j < top_k; j += 32) { const int c = ir[j]; wr[j] = c >= 0 ? expf(lr[c] - mx) / sum : 0.f; }
  if (top_k > 32) __syncwarp();  // rounds >= 32: their ir / wr entries are read back below
  if (wd) {
    for (int c0 = 0; c0 < C; c0 += 32) {
      const int c = c0 + lane;
      float val = 0.f;
      for (int j = 0; j < min(top_k, 32); ++j) {
        const int cj = __shfl_sync(0xffffffffu, mine, j);
        const float wj = __shfl_sync(0xffffffffu, wmine, j);
        if (cj == c) val = wj;
      }
      for (int j = 32; j < top_k; ++j)
        if (ir[j] == c) val = wr[j];
      if (c < C) wd[c] = val;
    }
  }
  if (top_k > 32) __syncwarp();
  for (int j = lane; j < k_out; j += 32) {
    if (j < 32) {
      ir[j] = (skip || j >= top_k) ? -1 : mine;
      wr[j] = (skip || j >= top_k) ? 0.f : wmine;
    } else if (skip || j >= top_k) {
      ir[j] = -1;
      wr[j] = 0.f;
    }
  }
}

// One warp per row; dynamic smem: TOPK_WARPS * C floats.
__global__ void __launch_bounds__(TOPK_WARPS * 32) route_topk_kernel(
    const float* __restrict__ logit, int64_t n_rows, int C, const int32_t* __restrict__ n_chunks_of,
    int64_t rows_per_lib, int top_k, int k_out, const float* __restrict__ row_w, int32_t* __restrict__ idx,
    float* __restrict__ wk, float* __restrict__ w_dense) {
  extern __shared__ float sv_all[];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * TOPK_WARPS + w;
  if (row >= n_rows) return;
  const int64_t lib = row / rows_per_lib;
  const int nc = n_chunks_of ? min(n_chunks_of[lib], C) : C;
  topk_row(logit + row * C, sv_all + (int64_t)w * C, C, nc, top_k, k_out, row_w ? row_w[row] : 1.f,
           idx + row * k_out, wk + row * k_out, w_dense ? w_dense + row * C : nullptr, lane);
}

// Decode: the input projection's row pass (project.cuh) and the routing of the same row in one CTA per row, so q
// never leaves the CTA between the two: the row's summary keys are requested from HBM before the wait for the
// GEMM (Library data that no kernel of the step writes), q is kept in shared memory once normalised, each warp
// takes the dot products of chunks w, w + n_warps, ... with the S rows now in L2 (route_dot: the same sums in
// the same order as route_fused_kernel), and warp 0 runs topk_row. Dynamic smem: q [d_s], the logits [C] and the
// top-k scratch [C] floats.
struct RouteFuse {
  const float* S;
  int C;
  const int32_t* n_chunks_of;
  int64_t rows_per_lib;
  float temp;
  int top_k, k_out;
  const float* row_w;
  int32_t* idx;
  float* wk;
  float* w_dense;
  float* logit_out;
  // With gridDim.y = G > 1 CTAs per row: the row's logits pass through xlg [n_rows, C] (global), and done[row]
  // (zeroed by the projection GEMM of the same call) counts the CTAs that stored theirs.
  float* xlg;
  int* done;
  // dense shard routing instead of the top-k (non-null): route_lse_kernel's output, w_dense = e^(l - max) and
  // lse_header[4 row] = (max, sum, 0, 0)
  float* lse_header;
};

// Grid (n_rows, G). CTA (row, g) computes the row's q (every CTA the same values; only g = 0 writes q, 1/rms, the
// gate and the selector logits) and the dot products of chunks [g * per, (g + 1) * per), per = ceil(C / G): the
// row's summary keys stream through G SMs instead of one. With G > 1 each CTA stores its logits in xlg, and the
// CTA that counts last in done[row] (after a fence) reads the whole row back and runs the top-k (or, for dense
// shard routing, route_lse_kernel's max / sum and unnormalised weights).
template <typename TH, int VPT>
__global__ void __launch_bounds__(ROW_THREADS) project_in_route_kernel(const TH* __restrict__ h, const PinArgs a,
                                                                      const RouteFuse rf) {
  extern __shared__ float pr_sh[];
  __shared__ float2 red2[32];
  __shared__ float red[32];
  __shared__ float zsh[32];
  __shared__ int last_sh;
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int G = (int)gridDim.y, g = (int)blockIdx.y;
  const int64_t lib = row / rf.rows_per_lib;
  const int nc = rf.n_chunks_of ? min(rf.n_chunks_of[lib], rf.C) : rf.C;
  const int per = (rf.C + G - 1) / G;
  const int c_lo = g * per, c_hi = min(rf.C, c_lo + per);
  const float* s_lib = rf.S + lib * rf.C * (int64_t)a.d_s;
  for (int c = c_lo + (int)threadIdx.x; c < min(c_hi, nc); c += blockDim.x)
    prefetch_l2_bulk(s_lib + (int64_t)c * a.d_s, (uint32_t)a.d_s * 4u);
  const float2 pre = pin_row_pre<TH>(h + row * a.d_m, a, zsh, g == 0);
  pdl_wait();
  float4 o[VPT];
  int n[VPT];
  bool ok[VPT];
  pin_row_post<VPT>(a, row, pre, zsh, red2, red, o, n, ok, g == 0);
  float* qs = pr_sh;
  float* lg = pr_sh + a.d_s;
#pragma unroll
  for (int q = 0; q < VPT; ++q)
    if (ok[q]) *reinterpret_cast<float4*>(qs + n[q]) = o[q];
  __syncthreads();
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float* xr = G > 1 ? rf.xlg + row * rf.C : nullptr;
  for (int c = c_lo + w; c < c_hi; c += nw) {
    float l = -CUDART_INF_F;
    if (c < nc) l = route_dot(qs, s_lib + (int64_t)c * a.d_s, a.d_s, lane) * rf.temp;
    if (lane == 0) {
      if (xr) xr[c] = l;
      else lg[c] = l;
      if (rf.logit_out && rf.logit_out != rf.xlg) rf.logit_out[row * rf.C + c] = l;
    }
  }
  __syncthreads();
  if (G > 1) {
    if (threadIdx.x == 0) {
      __threadfence();  // this CTA's logits (ordered before by the barrier) become visible before the count
      last_sh = atomicAdd(rf.done + row, 1) == G - 1;
      if (last_sh) __threadfence();
    }
    __syncthreads();
    if (!last_sh) return;
    for (int c = threadIdx.x; c < rf.C; c += blockDim.x) lg[c] = __ldcg(xr + c);
    __syncthreads();
  }
  if (w != 0) return;
  if (rf.lse_header) {  // route_lse_kernel's arithmetic, in its order, on the row's logits
    float mx = -CUDART_INF_F;
    for (int c = lane; c < nc; c += 32) mx = fmaxf(mx, lg[c]);
    mx = warp_max(mx);
    float sum = 0.f;
    if (nc > 0)
      for (int c = lane; c < nc; c += 32) sum += expf(lg[c] - mx);
    sum = warp_sum(sum);
    float* wr = rf.w_dense + row * rf.C;
    for (int c = lane; c < rf.C; c += 32) wr[c] = c < nc ? expf(lg[c] - mx) : 0.f;
    if (lane == 0) {
      rf.lse_header[row * 4] = mx;
      rf.lse_header[row * 4 + 1] = sum;
      rf.lse_header[row * 4 + 2] = 0.f;
      rf.lse_header[row * 4 + 3] = 0.f;
    }
    return;
  }
  topk_row(lg, lg + rf.C, rf.C, nc, rf.top_k, rf.k_out, rf.row_w ? rf.row_w[row] : 1.f, rf.idx + row * rf.k_out,
           rf.wk + row * rf.k_out, rf.w_dense ? rf.w_dense + row * rf.C : nullptr, lane);
}

// Decode routing in one launch: a cluster of RF_CL CTAs (RF_CL * 8 warps) takes `rpc` consecutive rows. Its warps
// share the rpc * C dot products (route_dot, the same sums as route_logits_kernel), and each writes its logit
// into the leader CTA's shared memory; after the cluster barrier the leader's warp r runs topk_row on row r.
// Dynamic smem: the rpc q rows (rpc * d_s floats, every CTA), then 2 * rpc * C floats (the logits and the top-k
// scratch, used in the leader CTA only).
constexpr int RF_CL = 8;
__global__ void __cluster_dims__(RF_CL, 1, 1) __launch_bounds__(256) route_fused_kernel(
    const float* __restrict__ q, int64_t n_rows, int d_s, const float* __restrict__ S, int C,
    const int32_t* __restrict__ n_chunks_of, int64_t rows_per_lib, float temp, int rpc, int top_k, int k_out,
    const float* __restrict__ row_w, int32_t* __restrict__ idx, float* __restrict__ wk, float* __restrict__ w_dense,
    float* __restrict__ logit_out) {
  extern __shared__ float rf_sh[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)(blockIdx.x / RF_CL) * rpc;
  float* lg_sh = rf_sh + (int64_t)rpc * d_s;  // after the staged q rows: logits, then the top-k scratch
  float* lead = cluster.map_shared_rank(lg_sh, 0);
  // The leader's shared memory may be written only once every CTA of the cluster runs: arrive now, wait after the
  // first dot product (its loads are in flight meanwhile).
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  {
    // Launched with programmatic serialisation: the S rows of this warp's dot products (Library data that no kernel
    // of the step writes) are requested from HBM before the wait for q, so they stream in while the input
    // projection finishes.
    for (int t = rank * 8 + w; t < rpc * C; t += RF_CL * 8) {
      const int r = t / C, c = t - r * C;
      const int64_t row = row0 + r;
      if (row >= n_rows) break;
      const int64_t lib = row / rows_per_lib;
      if (c >= (n_chunks_of ? min(n_chunks_of[lib], C) : C)) continue;
      const float* sr = S + (lib * C + c) * (int64_t)d_s;
      if ((d_s & 3) == 0) {
        if (lane == 0) prefetch_l2_bulk(sr, (uint32_t)d_s * 4u);
      } else {
        prefetch_row_l2(sr, d_s, lane);
      }
    }
    pdl_wait();
    const int64_t n_q = (min(n_rows, row0 + rpc) - row0) * (int64_t)d_s;
    for (int64_t i = threadIdx.x; i < n_q; i += blockDim.x) rf_sh[i] = q[row0 * d_s + i];
    __syncthreads();
  }
  bool started = false;
  const int n_dots = rpc * C;
  for (int t = rank * 8 + w; t < n_dots; t += RF_CL * 8) {
    const int r = t / C, c = t - r * C;
    const int64_t row = row0 + r;
    if (row >= n_rows) break;  // t only grows, and so does its row
    const int64_t lib = row / rows_per_lib;
    const int nc = n_chunks_of ? min(n_chunks_of[lib], C) : C;
    float l = -CUDART_INF_F;
    if (c < nc) l = route_dot(rf_sh + (int64_t)r * d_s, S + (lib * C + c) * (int64_t)d_s, d_s, lane) * temp;
    if (!started) {
      asm volatile("barrier.cluster.wait;" ::: "memory");
      started = true;
    }
    if (lane == 0) {
      lead[t] = l;
      if (logit_out) logit_out[row * C + c] = l;
    }
  }
  if (!started) asm volatile("barrier.cluster.wait;" ::: "memory");
  cluster.sync();  // every logit is in the leader's shared memory
  if (rank != 0 || w >= rpc) return;
  const int64_t row = row0 + w;
  if (row >= n_rows) return;
  const int64_t lib = row / rows_per_lib;
  const int nc = n_chunks_of ? min(n_chunks_of[lib], C) : C;
  topk_row(lg_sh + (int64_t)w * C, lg_sh + (int64_t)(rpc + w) * C, C, nc, top_k, k_out, row_w ? row_w[row] : 1.f,
           idx + row * k_out, wk + row * k_out, w_dense ? w_dense + row * C : nullptr, lane);
}

// Dense routing of a chunk shard, left unnormalised so that shards combine exactly: one warp per row turns the
// row's logits l_c (in w, overwritten in place) into e^(l_c - max) and writes the header (max, sum, 0, 0) at
// header[4 * row]. Chunks at or past the row's Library chunk count get weight 0; a row without chunks gets
// (-inf, 0), which the shard merge skips.
__global__ void __launch_bounds__(128) route_lse_kernel(float* __restrict__ w, int64_t n_rows, int C,
                                                       const int32_t* __restrict__ n_chunks_of, int64_t rows_per_lib,
                                                       float* __restrict__ header) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const int64_t lib = row / rows_per_lib;
  const int nc = n_chunks_of ? min(n_chunks_of[lib], C) : C;
  float* wr = w + row * C;
  float mx = -CUDART_INF_F;
  for (int c = lane; c < nc; c += 32) mx = fmaxf(mx, wr[c]);
  mx = warp_max(mx);
  float sum = 0.f;
  if (nc > 0)
    for (int c = lane; c < nc; c += 32) sum += expf(wr[c] - mx);
  sum = warp_sum(sum);
  for (int c = lane; c < C; c += 32) wr[c] = c < nc ? expf(wr[c] - mx) : 0.f;
  if (lane == 0) {
    header[row * 4] = mx;
    header[row * 4 + 1] = sum;
    header[row * 4 + 2] = 0.f;
    header[row * 4 + 3] = 0.f;
  }
}

// LayerSelector weights: one warp per row, lane = candidate (n_cand <= 32).
__global__ void __launch_bounds__(128) selector_weights_kernel(const float* __restrict__ z, int64_t n_rows,
                                                              int n_cand, int k, int straight_through,
                                                              float* __restrict__ w_out) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const float x = lane < n_cand ? z[row * n_cand + lane] : -CUDART_INF_F;
  float cur = lane < n_cand ? x : -CUDART_INF_F;
  bool kept = false;
  float vmax = -CUDART_INF_F;
  for (int t = 0; t < k; ++t) {
    float bv = cur;
    int bi = lane < n_cand ? lane : 0x7fffffff;
    warp_argmax(bv, bi);
    if (t == 0) vmax = bv;
    if (lane == bi) { kept = true; cur = -CUDART_INF_F; }
  }
  float e = 0.f;
  if (kept) e = straight_through ? 1.f : expf(x - vmax);
  const float sum = warp_sum(e);
  if (lane < n_cand) w_out[row * n_cand + lane] = kept ? (straight_through ? 1.f / (float)k : e / sum) : 0.f;
}

// Selector logits: one CTA per row; x = rms_norm(h) (rms != 0) or h; one warp per candidate dot product.
template <typename TH>
__global__ void __launch_bounds__(256) selector_logits_kernel(const TH* __restrict__ h, int d_m,
                                                             const float* __restrict__ u_w,
                                                             const float* __restrict__ u_b, int n_cand, int rms,
                                                             float eps, float* __restrict__ z_out) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const TH* hr = h + row * d_m;
  float scale = 1.f;
  if (rms) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < d_m; i += blockDim.x) { const float x = to_f32(hr[i]); ss = fmaf(x, x, ss); }
    ss = block_sum(ss, red);
    scale = rsqrtf(ss / (float)d_m + eps);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int c = wid; c < n_cand; c += nw) {
    const float* u = u_w + (int64_t)c * d_m;
    float d = 0.f;
    for (int i = lane; i < d_m; i += 32) d = fmaf(to_f32(hr[i]), u[i], d);
    d = warp_sum(d);
    if (lane == 0) z_out[row * n_cand + c] = d * scale + (u_b ? u_b[c] : 0.f);
  }
}

// S[lib, c] = L2(mean of the valid rows); one CTA per (lib, chunk), columns strided over threads.
template <typename T>
__global__ void __launch_bounds__(256) summaries_kernel(const T* __restrict__ slots, int64_t n_pages,
                                                       int64_t page_stride,
                                                       int page_rows, const int32_t* __restrict__ page_of,
                                                       const int32_t* __restrict__ n_valid, int C, int d_s,
                                                       float* __restrict__ S) {
  __shared__ float red[32];
  const int64_t lc = blockIdx.x;  // lib * C + c
  const int64_t page = page_of[lc];
  int nv = n_valid[lc];
  if (page < 0 || page >= n_pages) {  // never read outside the pool
    if (threadIdx.x == 0) flag_error(XENCB_DEV_BADPAGE);
    nv = 0;
  }
  nv = nv < 0 ? 0 : (nv > page_rows ? page_rows : nv);
  const T* base = slots + (nv > 0 ? page : 0) * page_stride;
  float* out = S + lc * (int64_t)d_s;
  const float cnt = (float)(nv > 0 ? nv : 1);
  float ss = 0.f;
  for (int j = threadIdx.x; j < d_s; j += blockDim.x) {
    float s = 0.f;
    for (int n = 0; n < nv; ++n) s += to_f32(base[(int64_t)n * d_s + j]);
    const float m = s / cnt;
    out[j] = m;
    ss = fmaf(m, m, ss);
  }
  ss = block_sum(ss, red);
  const float den = sqrtf(ss) + 1e-6f;
  for (int j = threadIdx.x; j < d_s; j += blockDim.x) out[j] = out[j] / den;
}

}  // namespace xencb

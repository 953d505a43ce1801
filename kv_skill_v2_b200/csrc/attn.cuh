// Attention diagnostics of LibraryInjector._branch, for one Library view (page table of the row's Library):
//
// record_attn (xenc/injector.py:259-260): the route-weighted slot attention of one query row,
//     aw[c, n] = w_c * softmax_n(read_temp * q . k_cn)        over the n_valid[c] rows of chunk c   (softmax read)
//              = w_c * (q . k_cn) / sqrt(max(n_valid[c], 1))                                        (linear read)
//   0 for chunks the row was not routed to (w_c = 0) and for rows past n_valid. One CTA per chunk; the scores in
//   fp32 from the slot type (the reference upcasts its slots), one warp per slot row.
//
// force_attn (xenc/injector.py:246-258): a given addressing fa [C, N] replaces aw for every token,
//     r1 = sum_{c, n < n_valid[c]} fa[c, n] v_cn         (rows past n_valid hold zeros in the reference's K)
//     r_t = s_t r1,  s_t = ||r0_t|| / (||fa @ K|| + 1e-6) with force_norm_match (r0 = aw @ K, the ordinary read),
//                    s_t = 1 otherwise.
//   forced_partial_kernel sums each chunk's weighted rows into a per-chunk partial (CTA per (chunk, 1024
//   columns)); forced_rows_kernel adds the partials in chunk order for each token row and applies s_t.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace xencb {

constexpr int AT_THREADS = 256;

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = is_max ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = is_max ? -CUDART_INF_F : 0.f;
  for (int i = 0; i < nw; ++i) t = is_max ? fmaxf(t, red[i]) : t + red[i];
  return t;
}

// Dynamic smem: q [d_s] then the scores [page_rows].
template <typename T>
__global__ void __launch_bounds__(AT_THREADS) read_attn_kernel(const float* __restrict__ q, int d_s,
                                                               const char* __restrict__ slots, int64_t n_pages,
                                                               int64_t page_stride_bytes, int page_rows,
                                                               const int32_t* __restrict__ page_of,
                                                               const int32_t* __restrict__ n_valid,
                                                               const int32_t* __restrict__ idx,
                                                               const float* __restrict__ wk, int k, float read_temp,
                                                               int softmax, float* __restrict__ out) {
  extern __shared__ float at_sh[];
  __shared__ float red[32];
  float* qs = at_sh;
  float* sc = at_sh + d_s;
  const int c = blockIdx.x;
  float w = 0.f;
  for (int j = 0; j < k; ++j)
    if (idx[j] == c && wk[j] != 0.f) w = wk[j];
  float* o = out + (int64_t)c * page_rows;
  const int64_t page = page_of[c];
  int nv = n_valid[c];
  if (nv > page_rows) { nv = page_rows; flag_error(XENCB_DEV_CLAMPED); }
  if (nv < 0) nv = 0;
  const bool bad = page < 0 || page >= n_pages;
  if (w != 0.f && bad) flag_error(XENCB_DEV_BADPAGE);
  if (w == 0.f || bad || nv == 0) {
    for (int n = threadIdx.x; n < page_rows; n += blockDim.x) o[n] = 0.f;
    return;
  }
  for (int i = threadIdx.x; i < d_s; i += blockDim.x) qs[i] = q[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const T* base = reinterpret_cast<const T*>(slots + page * page_stride_bytes);
  for (int n = warp; n < nv; n += nw) {
    const T* kr = base + (int64_t)n * d_s;
    float d = 0.f;
    for (int i = lane; i < d_s; i += 32) d = fmaf(qs[i], to_f32(kr[i]), d);
    d = warp_sum(d);
    if (lane == 0) sc[n] = d;
  }
  __syncthreads();
  if (softmax) {
    float m = -CUDART_INF_F;
    for (int n = threadIdx.x; n < nv; n += blockDim.x) m = fmaxf(m, sc[n] * read_temp);
    m = block_reduce(m, red, true);
    float l = 0.f;
    for (int n = threadIdx.x; n < nv; n += blockDim.x) l += expf(sc[n] * read_temp - m);
    l = block_reduce(l, red, false);
    for (int n = threadIdx.x; n < page_rows; n += blockDim.x)
      o[n] = n < nv ? w * (expf(sc[n] * read_temp - m) / l) : 0.f;
  } else {
    const float den = sqrtf((float)nv);
    for (int n = threadIdx.x; n < page_rows; n += blockDim.x) o[n] = n < nv ? w * (sc[n] / den) : 0.f;
  }
}

// part[c][col] = sum_{n < n_valid[c]} fa[c, n] * v_cn[col]; grid (C, ceil(d_s / (4 * AT_THREADS))).
template <typename T>
__global__ void __launch_bounds__(AT_THREADS) forced_partial_kernel(const float* __restrict__ fa, int d_s,
                                                                    const char* __restrict__ pool, int64_t n_pages,
                                                                    int64_t page_stride_bytes, int page_rows,
                                                                    const int32_t* __restrict__ page_of,
                                                                    const int32_t* __restrict__ n_valid,
                                                                    float* __restrict__ part) {
  const int c = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  const int64_t page = page_of[c];
  int nv = n_valid[c];
  nv = nv > page_rows ? page_rows : (nv < 0 ? 0 : nv);
  float a[4] = {0.f, 0.f, 0.f, 0.f};
  if (page < 0 || page >= n_pages) {
    if (threadIdx.x == 0 && blockIdx.y == 0) flag_error(XENCB_DEV_BADPAGE);
    nv = 0;
  }
  const T* base = reinterpret_cast<const T*>(pool + (nv ? page * page_stride_bytes : 0));
  const float* fr = fa + (int64_t)c * page_rows;
  for (int n = 0; n < nv; ++n) {
    const float f = fr[n];
    if (f == 0.f || col >= d_s) continue;
    const T* vr = base + (int64_t)n * d_s + col;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (col + e < d_s) a[e] = fmaf(f, to_f32(vr[e]), a[e]);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (col + e < d_s) part[(int64_t)c * d_s + col + e] = a[e];
}

// r_out[t] = s_t * sum_c part_v[c] (chunk order); s_t from ||r0_t|| and ||sum_c part_k[c]|| when r0 is given.
__global__ void __launch_bounds__(AT_THREADS) forced_rows_kernel(const float* __restrict__ part_v,
                                                                 const float* __restrict__ part_k, int C, int d_s,
                                                                 const float* __restrict__ r0,
                                                                 float* __restrict__ r_out,
                                                                 float* __restrict__ scale_out) {
  __shared__ float red[32];
  const int64_t t = blockIdx.x;
  float s = 1.f;
  if (r0) {
    float kk = 0.f, rr = 0.f;
    for (int col = threadIdx.x; col < d_s; col += blockDim.x) {
      float v = 0.f;
      for (int c = 0; c < C; ++c) v += part_k[(int64_t)c * d_s + col];
      kk = fmaf(v, v, kk);
      const float x = r0[t * d_s + col];
      rr = fmaf(x, x, rr);
    }
    kk = block_reduce(kk, red, false);
    rr = block_reduce(rr, red, false);
    s = sqrtf(rr) / (sqrtf(kk) + 1e-6f);
  }
  for (int col = threadIdx.x; col < d_s; col += blockDim.x) {
    float v = 0.f;
    for (int c = 0; c < C; ++c) v += part_v[(int64_t)c * d_s + col];
    r_out[t * d_s + col] = s * v;
  }
  if (scale_out && threadIdx.x == 0) scale_out[t] = s;
}

}  // namespace xencb

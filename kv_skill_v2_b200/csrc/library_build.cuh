// Library build on the device: the doc cache's ragged chunk rows -> a padded slot page per chunk, its valid-row
// count and its summary key, in two launches.
//
// Replaces the per-chunk host loop of Library.__init__ (xenc/library.py:47-67: pad each chunk's rows into
// K[c, :n_c], zeros after, optional centering K = L2(K - mu) on the valid rows only) and Library._summaries
// (xenc/library.py:69-74: S[c] = L2(sum of the valid rows / max(n_c, 1))).
//
// library_build_kernel: grid (chunk, split); each split owns a contiguous range of the page's rows and one CTA
//   spans the columns (8 per thread). Every valid row is read from HBM once, centred and normalised in
//   registers, written to its slot and added, as float32, into the thread's column sums (registers, fixed row
//   order). Padding rows are written as zeros. Each CTA stores its column sums into its slice of the workspace:
//   the summation order is fixed, so S is deterministic.
// library_summaries_kernel: one CTA per chunk sums the splits in order, divides by max(n_c, 1), normalises,
//   and stores S[c] and n_valid[c]. S is computed from the float32 values before they are rounded to the slot
//   type, as the reference computes it from its float32 Library.
// Bound: HBM (rows read once from DRAM, slots written once); a one-time build per Library.
#pragma once

#include "common.cuh"

namespace xencb {

constexpr int LB_VEC = 8;            // elements per thread per row (16 bytes of f16 / bf16, 32 bytes of f32)
constexpr int LB_ROWS = 8;           // rows per batch
constexpr int LB_MAX_THREADS = 512;  // d_s <= 4096

struct LibBuildArgs {
  const void* rows;
  int64_t n_rows_total;
  const int64_t* row_start;  // [n_chunks + 1]
  int n_chunks, d_s;
  const float* mu;           // [d_s] or nullptr
  void* slots;
  int64_t n_pages, page_stride;  // page_stride in elements
  int page_rows;
  const int32_t* page_of;
  int n_split, split_rows;
  float* part;               // [n_chunks][n_split][d_s]
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* out) {
  if constexpr (sizeof(T) == 4) {
    const uint4 a = *reinterpret_cast<const uint4*>(p), b = *reinterpret_cast<const uint4*>(p + 4);
    unpack16<float>(a, out);
    unpack16<float>(b, out + 4);
  } else {
    unpack16<T>(*reinterpret_cast<const uint4*>(p), out);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float* v) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    alignas(16) T h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(h);
  }
}

// The chunk's row range, checked against the row buffer; count clamped to the page. Flags are raised by the
// (chunk, split 0) CTA only, so each problem is reported once.
__device__ __forceinline__ int lb_chunk_rows(const LibBuildArgs& a, int c, int64_t* r0_out, bool report) {
  const int64_t r0 = a.row_start[c], r1 = a.row_start[c + 1];
  *r0_out = r0;
  if (r0 < 0 || r1 < r0 || r1 > a.n_rows_total) {
    if (report) flag_error(XENCB_DEV_BADROWS);
    return 0;
  }
  int64_t n = r1 - r0;
  if (n > a.page_rows) {
    if (report) flag_error(XENCB_DEV_CLAMPED);
    n = a.page_rows;
  }
  return (int)n;
}

// One CTA covers a row's columns: thread t owns columns [8t, 8t + 8) of every row in the CTA's range, so its
// column sums and its slice of mu stay in registers. Rows go in batches of LB_ROWS, all loaded before first use
// (LB_ROWS 16-byte loads in flight per thread); a centred batch needs one block reduction of LB_ROWS squared
// norms (double-buffered partials: one barrier per batch).
template <typename TI, typename TO>
__global__ void __maxnreg__(80) library_build_kernel(const LibBuildArgs a) {
  __shared__ float red[2][LB_MAX_THREADS / 32][LB_ROWS];
  static_assert(LB_ROWS == 8, "the norm reduce-scatter below is written for 8 rows per batch");
  const int d_s = a.d_s;
  const int c = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int j = threadIdx.x * LB_VEC;
  const bool col_ok = j < d_s;
  const bool report = split == 0 && threadIdx.x == 0;
  int64_t r0;
  const int count = lb_chunk_rows(a, c, &r0, report);
  const int64_t page = a.page_of[c];
  const bool page_ok = page >= 0 && page < a.n_pages;
  if (!page_ok && report) flag_error(XENCB_DEV_BADPAGE);
  TO* pbase = static_cast<TO*>(a.slots) + (page_ok ? page : 0) * a.page_stride + j;
  const TI* src = static_cast<const TI*>(a.rows) + r0 * (int64_t)d_s + j;
  const int s0 = split * a.split_rows;
  const int s1 = min(a.page_rows, s0 + a.split_rows);
  const bool center = a.mu != nullptr;
  float m[LB_VEC], cs[LB_VEC];
#pragma unroll
  for (int i = 0; i < LB_VEC; ++i) {
    m[i] = center && col_ok ? __ldg(a.mu + j + i) : 0.f;
    cs[i] = 0.f;
  }
  constexpr int W = sizeof(TI) == 4 ? 2 : 1;  // 16-byte words per 8 elements
  int buf = 0;
  for (int rb = s0; rb < s1; rb += LB_ROWS) {
    const int nvalid = max(0, min(LB_ROWS, min(count, s1) - rb));  // valid rows of this batch (uniform)
    uint4 v[LB_ROWS][W];
#pragma unroll
    for (int i = 0; i < LB_ROWS; ++i) {
      if (i < nvalid && col_ok) {
#pragma unroll
        for (int w = 0; w < W; ++w) v[i][w] = __ldcs(reinterpret_cast<const uint4*>(src + (int64_t)(rb + i) * d_s) + w);
      }
    }
    float inv[LB_ROWS];
#pragma unroll
    for (int i = 0; i < LB_ROWS; ++i) inv[i] = 1.f;
    if (center && nvalid > 0) {
      float ss[LB_ROWS];
#pragma unroll
      for (int i = 0; i < LB_ROWS; ++i) {
        ss[i] = 0.f;
        if (i < nvalid && col_ok) {
          float x[LB_VEC];
          if constexpr (W == 2) { unpack16<float>(v[i][0], x); unpack16<float>(v[i][1], x + 4); }
          else unpack16<TI>(v[i][0], x);
#pragma unroll
          for (int e = 0; e < LB_VEC; ++e) {
            const float t = x[e] - m[e];
            ss[i] = fmaf(t, t, ss[i]);
          }
        }
      }
      // butterfly reduce-scatter of the 8 row sums over the warp: 4 + 2 + 1 + 2 shuffles; lane l ends with the
      // warp total of row 4*b4 + 2*b3 + b2 (b = bits of l)
      const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4;
      float k4[4], k2[2];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        k4[i] = (h4 ? ss[i + 4] : ss[i]) + __shfl_xor_sync(0xffffffffu, h4 ? ss[i] : ss[i + 4], 16);
#pragma unroll
      for (int i = 0; i < 2; ++i)
        k2[i] = (h3 ? k4[i + 2] : k4[i]) + __shfl_xor_sync(0xffffffffu, h3 ? k4[i] : k4[i + 2], 8);
      float t = (h2 ? k2[1] : k2[0]) + __shfl_xor_sync(0xffffffffu, h2 ? k2[0] : k2[1], 4);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      if ((lane & 3) == 0) red[buf][warp][lane >> 2] = t;
      __syncthreads();
      // lanes 0..7 total row `lane` over the warps (fixed order), then broadcast the 8 scales
      float tot = 0.f;
      if (lane < LB_ROWS)
        for (int w = 0; w < nw; ++w) tot += red[buf][w][lane];
      // x / (|x| + eps) as one correctly rounded reciprocal and a multiply per element
      const float my_inv = __frcp_rn(sqrtf(tot) + 1e-6f);
#pragma unroll
      for (int i = 0; i < LB_ROWS; ++i) inv[i] = __shfl_sync(0xffffffffu, my_inv, i);
      buf ^= 1;
    }
#pragma unroll
    for (int i = 0; i < LB_ROWS; ++i) {
      const int r = rb + i;
      if (r >= s1 || !col_ok) continue;
      TO* dst = pbase + (int64_t)r * d_s;
      if (i < nvalid) {
        float x[LB_VEC];
        if constexpr (W == 2) { unpack16<float>(v[i][0], x); unpack16<float>(v[i][1], x + 4); }
        else unpack16<TI>(v[i][0], x);
        if (center) {
#pragma unroll
          for (int e = 0; e < LB_VEC; ++e) x[e] = (x[e] - m[e]) * inv[i];
        }
        if (page_ok) store8<TO>(dst, x);
#pragma unroll
        for (int e = 0; e < LB_VEC; ++e) cs[e] += x[e];
      } else if (page_ok) {
        const float z[LB_VEC] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        store8<TO>(dst, z);
      }
    }
  }
  if (col_ok) {
    float* out = a.part + ((int64_t)c * a.n_split + split) * d_s + j;
    *reinterpret_cast<float4*>(out) = make_float4(cs[0], cs[1], cs[2], cs[3]);
    *reinterpret_cast<float4*>(out + 4) = make_float4(cs[4], cs[5], cs[6], cs[7]);
  }
}

__global__ void __launch_bounds__(256) library_summaries_kernel(const LibBuildArgs a, int32_t* __restrict__ n_valid,
                                                                float* __restrict__ S) {
  __shared__ float red[32];
  const int c = blockIdx.x;
  int64_t r0;
  const int count = lb_chunk_rows(a, c, &r0, false);
  const float cnt = (float)(count > 0 ? count : 1);
  const float* part = a.part + (int64_t)c * a.n_split * a.d_s;
  float ss = 0.f;
  float* out = S ? S + (int64_t)c * a.d_s : nullptr;
  for (int j = threadIdx.x; j < a.d_s; j += blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < a.n_split; ++p) s += part[(int64_t)p * a.d_s + j];
    const float m = s / cnt;
    if (out) out[j] = m;
    ss = fmaf(m, m, ss);
  }
  ss = block_sum(ss, red);
  if (out) {
    const float den = sqrtf(ss) + 1e-6f;
    for (int j = threadIdx.x; j < a.d_s; j += blockDim.x) out[j] = out[j] / den;
  }
  if (n_valid && threadIdx.x == 0) n_valid[c] = count;
}

}  // namespace xencb

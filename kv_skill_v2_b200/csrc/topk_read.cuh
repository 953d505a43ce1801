// D8 top-k slot selection and the read over the selected slots (xenc/topk_read.py).
//
// select_scores_kernel  (TopKSelector.head_scores + pool_scores, xenc/topk_read.py:215-239)
//   s[r, slot] = pool_h pool_t (q[r, t, h] . keys[slot, h / groups])   (GQA: query head h scores KV head h/groups)
//   pool_t: the one position given (query "last"), max ("all_max") or mean ("all_mean") over T positions;
//   pool_h: max or mean over the n_q heads; slots that are not valid (n >= n_valid of the chunk, or a chunk past
//   the Library's count) get -inf. Keys are [C * page_rows, n_kv * hd] per Library (the selection keys laid out
//   on the residual Library's pages), float32 or float16. Grid (32-slot tiles, rows); warp w takes KV heads
//   w, w + 8, ...; lane = slot; q is read with warp-uniform addresses (L1 broadcasts).
//   Bound: HBM (keys read once per query row) or FMA issue, whichever is larger (about 2 FMA per key byte).
// select_topk_kernel  (TopKSelector.select_from_input: sc.topk(k), :251-254)
//   One CTA per row: radix select of the k-th largest score (4 passes of 8-bit histograms over orderable keys),
//   an index-ordered compaction (ties at the threshold: lower slot first), then a bitonic sort of the k winners by
//   (score desc, slot asc). Outputs idx [r, k] int32 and the k scores.
// topk_read_kernel  (TopKLibraryInjector._branch, :392-413)
//   a = q . K[idx] (k selected slots), softmax(a * read_temp) over the k (or a / sqrt(k)), r = a @ V[idx].
//   Grid (idx sets, query-row blocks of TR rows); the block's query rows sit in shared memory; warps score the
//   selected rows (one row per warp at a time), warps 0..TR-1 finish one query row's softmax each, then each
//   thread owns 8 columns and sums the selected value rows. Slot s of set b is row s % page_rows of page
//   page_of[lib, s / page_rows] (lib = b when there are several Libraries, else 0).
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace xencb {

constexpr int SEL_THREADS = 256;
constexpr int SEL_TILE = 32;        // slots per CTA
constexpr int SEL_MAX_G = 16;       // GQA group size supported
constexpr int SEL_MAX_KV = 64;
constexpr int TOPK_THREADS = 1024;
constexpr int TOPK_MAX_K = 2048;
constexpr int TR_ROWS = 8;          // query rows per topk_read CTA
constexpr int TR_THREADS = 256;

struct SelectArgs {
  const float* q;          // [R, T, n_q, hd]
  int64_t n_rows;
  int T, n_q, n_kv, hd;
  const void* keys;        // per Library [C * page_rows, n_kv * hd]
  int64_t keys_lib_stride; // elements between Libraries
  int page_rows, n_chunks;
  const int32_t* n_valid;  // [n_lib, C]
  const int32_t* n_chunks_of;  // [n_lib] or nullptr
  int64_t rows_per_lib;
  int t_pool;              // 0 max, 1 mean (T == 1 for "last")
  int h_pool;              // 0 max, 1 mean
  float* scores;           // [R, C * page_rows]
};

template <typename TK>
__global__ void __launch_bounds__(SEL_THREADS) select_scores_kernel(const SelectArgs a) {
  __shared__ float red[SEL_MAX_KV][SEL_TILE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.y;
  const int64_t lib = row / a.rows_per_lib;
  const int S = a.n_chunks * a.page_rows;
  const int slot = blockIdx.x * SEL_TILE + lane;
  const int g = a.n_q / a.n_kv;
  const int d_k = a.n_kv * a.hd;
  const TK* kb = static_cast<const TK*>(a.keys) + lib * a.keys_lib_stride;
  const float* qrow = a.q + row * (int64_t)a.T * a.n_q * a.hd;

  for (int kv = warp; kv < a.n_kv; kv += SEL_THREADS / 32) {
    float hv[SEL_MAX_G];  // per head of the group, pooled over positions
#pragma unroll
    for (int i = 0; i < SEL_MAX_G; ++i) hv[i] = a.t_pool == 0 ? -CUDART_INF_F : 0.f;
    if (slot < S) {
      const TK* kr = kb + (int64_t)slot * d_k + kv * a.hd;
      for (int t = 0; t < a.T; ++t) {
        const float* qk = qrow + ((int64_t)t * a.n_q + kv * g) * a.hd;  // the group's heads at position t
        float acc[SEL_MAX_G];
#pragma unroll
        for (int i = 0; i < SEL_MAX_G; ++i) acc[i] = 0.f;
        for (int e = 0; e < a.hd; e += 8) {
          float kx[8];
          if constexpr (sizeof(TK) == 4) {
            unpack16<float>(__ldg(reinterpret_cast<const uint4*>(kr + e)), kx);
            unpack16<float>(__ldg(reinterpret_cast<const uint4*>(kr + e + 4)), kx + 4);
          } else {
            unpack16<TK>(__ldg(reinterpret_cast<const uint4*>(kr + e)), kx);
          }
#pragma unroll
          for (int hh = 0; hh < SEL_MAX_G; ++hh) {
            if (hh < g) {  // every lane reads the same q address: a broadcast
              const float4 q0 = __ldg(reinterpret_cast<const float4*>(qk + hh * a.hd + e));
              const float4 q1 = __ldg(reinterpret_cast<const float4*>(qk + hh * a.hd + e + 4));
              float sv = acc[hh];
              sv = fmaf(q0.x, kx[0], sv); sv = fmaf(q0.y, kx[1], sv); sv = fmaf(q0.z, kx[2], sv);
              sv = fmaf(q0.w, kx[3], sv); sv = fmaf(q1.x, kx[4], sv); sv = fmaf(q1.y, kx[5], sv);
              sv = fmaf(q1.z, kx[6], sv); sv = fmaf(q1.w, kx[7], sv);
              acc[hh] = sv;
            }
          }
        }
#pragma unroll
        for (int hh = 0; hh < SEL_MAX_G; ++hh)
          if (hh < g) hv[hh] = a.t_pool == 0 ? fmaxf(hv[hh], acc[hh]) : hv[hh] + acc[hh];
      }
    }
    float p = a.h_pool == 0 ? -CUDART_INF_F : 0.f;
#pragma unroll
    for (int hh = 0; hh < SEL_MAX_G; ++hh) {
      if (hh < g) {
        const float v = a.t_pool == 0 ? hv[hh] : hv[hh] / (float)a.T;
        p = a.h_pool == 0 ? fmaxf(p, v) : p + v;
      }
    }
    red[kv][lane] = p;
  }
  __syncthreads();
  if (warp == 0 && slot < S) {
    float p = a.h_pool == 0 ? -CUDART_INF_F : 0.f;
    for (int kv = 0; kv < a.n_kv; ++kv) {
      const float v = red[kv][lane];
      p = a.h_pool == 0 ? fmaxf(p, v) : p + v;
    }
    if (a.h_pool == 1) p /= (float)a.n_q;
    const int c = slot / a.page_rows, n = slot - c * a.page_rows;
    const int nc = a.n_chunks_of ? a.n_chunks_of[lib] : a.n_chunks;
    const bool valid = c < nc && n < a.n_valid[lib * a.n_chunks + c];
    a.scores[row * (int64_t)S + slot] = valid ? p : -CUDART_INF_F;
  }
}

// ------------------------------------------------------------------------------------------------ top-k
__device__ __forceinline__ uint32_t order_key(float x) {  // larger float -> larger unsigned key
  const uint32_t u = x == 0.f ? 0u : __float_as_uint(x);  // -0 and +0 compare equal, as floats do
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(TOPK_THREADS) select_topk_kernel(const float* __restrict__ scores, int S, int k,
                                                                   int32_t* __restrict__ idx_out,
                                                                   float* __restrict__ score_out) {
  __shared__ int hist[256];
  __shared__ int sh_bin, sh_rem;
  __shared__ int cnt_gt[TOPK_THREADS], cnt_eq[TOPK_THREADS];
  __shared__ uint32_t skey[TOPK_MAX_K];
  __shared__ int sidx[TOPK_MAX_K];
  const int tid = threadIdx.x;
  const float* sc = scores + (int64_t)blockIdx.x * S;

  // ---- radix select: the k-th largest key, 8 bits at a time from the top
  uint32_t prefix = 0, pmask = 0;
  int rem = k;  // how many of the remaining candidates (matching the prefix) are still to take
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += TOPK_THREADS) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < S; i += TOPK_THREADS) {
      const uint32_t key = order_key(sc[i]);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid < 32) {
      // scan bins from the top: lane l sums bins [255 - 8l - 7, 255 - 8l]
      int part = 0;
      for (int b = 0; b < 8; ++b) part += hist[255 - 8 * tid - b];
      int incl = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += v;
      }
      const int excl = incl - part;
      if (excl < rem && incl >= rem) {  // the bin holding the rem-th largest is in this lane's group
        int run = excl;
        for (int b = 0; b < 8; ++b) {
          const int bin = 255 - 8 * tid - b;
          if (run + hist[bin] >= rem) { sh_bin = bin; sh_rem = rem - run; break; }
          run += hist[bin];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sh_bin << shift;
    pmask |= 255u << shift;
    rem = sh_rem;
    __syncthreads();
  }
  const uint32_t thr = prefix;   // the k-th largest key; `rem` of the keys equal to it are taken
  const int take_eq = rem;

  // ---- index-ordered compaction: thread t scans slots [t * seg, (t + 1) * seg)
  const int seg = (S + TOPK_THREADS - 1) / TOPK_THREADS;
  const int i0 = tid * seg, i1 = min(S, i0 + seg);
  int ngt = 0, neq = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = order_key(sc[i]);
    ngt += key > thr;
    neq += key == thr;
  }
  cnt_gt[tid] = ngt;
  cnt_eq[tid] = neq;
  __syncthreads();
  // exclusive scans of both counts (Hillis-Steele over the block, in place, two arrays)
  for (int o = 1; o < TOPK_THREADS; o <<= 1) {
    const int a_gt = tid >= o ? cnt_gt[tid - o] : 0;
    const int a_eq = tid >= o ? cnt_eq[tid - o] : 0;
    __syncthreads();
    cnt_gt[tid] += a_gt;
    cnt_eq[tid] += a_eq;
    __syncthreads();
  }
  const int n_gt_total = cnt_gt[TOPK_THREADS - 1];
  int pos_gt = cnt_gt[tid] - ngt, pos_eq = cnt_eq[tid] - neq;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = order_key(sc[i]);
    if (key > thr) {
      skey[pos_gt] = key; sidx[pos_gt] = i; ++pos_gt;
    } else if (key == thr) {
      if (pos_eq < take_eq) { skey[n_gt_total + pos_eq] = key; sidx[n_gt_total + pos_eq] = i; }
      ++pos_eq;
    }
  }
  // pad to a power of two with keys that sort last
  int kp = 1;
  while (kp < k) kp <<= 1;
  for (int i = k + tid; i < kp; i += TOPK_THREADS) { skey[i] = 0u; sidx[i] = 0x7fffffff; }
  __syncthreads();
  // ---- bitonic sort, descending by key, ascending by slot on equal keys
  for (int size = 2; size <= kp; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < kp; i += TOPK_THREADS) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;  // this pair's run sorts "first before": larger key first
          const uint32_t ki = skey[i], kj = skey[j];
          const int xi = sidx[i], xj = sidx[j];
          const bool i_first = ki > kj || (ki == kj && xi < xj);
          if (up ? !i_first : i_first) {
            skey[i] = kj; skey[j] = ki; sidx[i] = xj; sidx[j] = xi;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < k; i += TOPK_THREADS) {
    idx_out[(int64_t)blockIdx.x * k + i] = sidx[i];
    if (score_out) score_out[(int64_t)blockIdx.x * k + i] = sc[sidx[i]];
  }
}

// ------------------------------------------------------------------------------------------------ read
struct TopkReadArgs {
  const float* q;          // [R, d_s]
  int64_t n_rows;
  int d_s;
  const char* slots;
  const char* vslots;      // untied values or nullptr
  int64_t n_pages, page_stride_bytes;
  int page_rows, n_chunks;
  const int32_t* page_of;  // [n_lib, C]
  int64_t n_lib;
  const int32_t* idx;      // [n_sets, k]
  int n_sets, k;
  int64_t rows_per_set;
  float qscale;            // read_temp * log2(e) (softmax) or 1
  int softmax;
  float* r_out;            // [R, d_s]
  float* attn_out;         // [R, k] or nullptr
};

template <typename T>
__global__ void __launch_bounds__(TR_THREADS) topk_read_kernel(const TopkReadArgs a) {
  extern __shared__ __align__(16) float tr_smem[];
  float* qs = tr_smem;                                   // [TR_ROWS][d_s]
  float* at = tr_smem + (size_t)TR_ROWS * a.d_s;         // [TR_ROWS][k]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int set = blockIdx.x;
  const int64_t t0 = (int64_t)blockIdx.y * TR_ROWS;
  const int64_t left = a.rows_per_set - t0;
  const int nt = left < TR_ROWS ? (int)left : TR_ROWS;
  if (nt <= 0) return;
  const int64_t row0 = (int64_t)set * a.rows_per_set + t0;
  const int64_t lib = a.n_lib > 1 ? set : 0;
  const int32_t* ix = a.idx + (int64_t)set * a.k;
  const int d_s = a.d_s;

  for (int j = threadIdx.x * 4; j < TR_ROWS * d_s; j += TR_THREADS * 4) {
    const int t = j / d_s;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < nt) v = *reinterpret_cast<const float4*>(a.q + (row0 + t) * d_s + (j - t * d_s));
    *reinterpret_cast<float4*>(qs + j) = v;
  }
  __syncthreads();

  // slot -> row address (invalid slots or pages read nothing and score -inf / 0)
  auto row_ptr = [&](const char* pool, int s) -> const T* {
    if (s < 0 || s >= a.n_chunks * a.page_rows) return nullptr;
    const int c = s / a.page_rows, n = s - c * a.page_rows;
    const int64_t page = a.page_of[lib * a.n_chunks + c];
    if (page < 0 || page >= a.n_pages) return nullptr;
    return reinterpret_cast<const T*>(pool + page * a.page_stride_bytes) + (int64_t)n * d_s;
  };

  // ---- scores
  for (int i = warp; i < a.k; i += TR_THREADS / 32) {
    const T* kr = row_ptr(a.slots, ix[i]);
    float dot[TR_ROWS];
#pragma unroll
    for (int t = 0; t < TR_ROWS; ++t) dot[t] = 0.f;
    if (kr) {
      for (int j = lane * 8; j < d_s; j += 256) {
        float kx[8];
        if constexpr (sizeof(T) == 4) {
          unpack16<float>(__ldg(reinterpret_cast<const uint4*>(kr + j)), kx);
          unpack16<float>(__ldg(reinterpret_cast<const uint4*>(kr + j + 4)), kx + 4);
        } else {
          unpack16<T>(__ldg(reinterpret_cast<const uint4*>(kr + j)), kx);
        }
#pragma unroll
        for (int t = 0; t < TR_ROWS; ++t) {
          const float4 q0 = *reinterpret_cast<const float4*>(qs + t * d_s + j);
          const float4 q1 = *reinterpret_cast<const float4*>(qs + t * d_s + j + 4);
          float s = dot[t];
          s = fmaf(q0.x, kx[0], s); s = fmaf(q0.y, kx[1], s); s = fmaf(q0.z, kx[2], s); s = fmaf(q0.w, kx[3], s);
          s = fmaf(q1.x, kx[4], s); s = fmaf(q1.y, kx[5], s); s = fmaf(q1.z, kx[6], s); s = fmaf(q1.w, kx[7], s);
          dot[t] = s;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TR_ROWS; ++t) {
      const float s = warp_sum(dot[t]);
      if (lane == 0) at[t * a.k + i] = kr ? s : -CUDART_INF_F;
    }
  }
  __syncthreads();
  // ---- per query row: softmax over the k scores (or the linear 1/sqrt(k) scale)
  if (warp < nt) {
    float* ar = at + warp * a.k;
    if (a.softmax) {
      // qscale = read_temp * log2(e): exp2 of the scaled, max-shifted scores
      float mx = -CUDART_INF_F;
      for (int i = lane; i < a.k; i += 32) mx = fmaxf(mx, ar[i] * a.qscale);
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sum = 0.f;
      for (int i = lane; i < a.k; i += 32) {
        const float e = ar[i] == -CUDART_INF_F ? 0.f : exp2f(ar[i] * a.qscale - mx);
        ar[i] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      const float inv = 1.f / sum;
      for (int i = lane; i < a.k; i += 32) ar[i] *= inv;
    } else {
      const float sc = rsqrtf((float)a.k);
      for (int i = lane; i < a.k; i += 32) ar[i] = ar[i] == -CUDART_INF_F ? 0.f : ar[i] * sc;
    }
    __syncwarp();
    if (a.attn_out)
      for (int i = lane; i < a.k; i += 32) a.attn_out[(row0 + warp) * a.k + i] = ar[i];
  }
  __syncthreads();
  // ---- r = a @ V over the selected rows: thread owns 8 columns (looping for d_s > 2048)
  const char* vpool = a.vslots ? a.vslots : a.slots;
  for (int j = threadIdx.x * 8; j < d_s; j += TR_THREADS * 8) {
    float acc[TR_ROWS][8];
#pragma unroll
    for (int t = 0; t < TR_ROWS; ++t)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[t][e] = 0.f;
    for (int i = 0; i < a.k; ++i) {
      const T* vr = row_ptr(vpool, ix[i]);
      if (!vr) continue;
      float vx[8];
      if constexpr (sizeof(T) == 4) {
        unpack16<float>(__ldg(reinterpret_cast<const uint4*>(vr + j)), vx);
        unpack16<float>(__ldg(reinterpret_cast<const uint4*>(vr + j + 4)), vx + 4);
      } else {
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(vr + j)), vx);
      }
#pragma unroll
      for (int t = 0; t < TR_ROWS; ++t) {
        const float w = at[t * a.k + i];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[t][e] = fmaf(w, vx[e], acc[t][e]);
      }
    }
#pragma unroll
    for (int t = 0; t < TR_ROWS; ++t) {
      if (t < nt) {
        float* o = a.r_out + (row0 + t) * d_s + j;
        *reinterpret_cast<float4*>(o) = make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(acc[t][4], acc[t][5], acc[t][6], acc[t][7]);
      }
    }
  }
}

}  // namespace xencb

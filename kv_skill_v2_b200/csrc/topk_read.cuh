// D8 top-k slot selection and the read over the selected slots (xenc/topk_read.py).
//
// select_scores_kernel  (TopKSelector.head_scores + pool_scores, xenc/topk_read.py:215-239)
//   s[r, slot] = pool_h pool_t (q[r, t, h] . keys[slot, h / groups])   (GQA: query head h scores KV head h/groups)
//   pool_t: the one position given (query "last"), max ("all_max") or mean ("all_mean") over T positions;
//   pool_h: max or mean over the n_q heads; slots that are not valid (n >= n_valid of the chunk, or a chunk past
//   the Library's count) get -inf. Keys are [C * page_rows, n_kv * hd] per Library (the selection keys laid out
//   on the residual Library's pages), float32 or float16. Grid (128-slot tiles, rows); warp w takes KV heads
//   w, w + 8, ...; lane l scores slots l + 32u (u < 4); q is read with warp-uniform addresses (L1 broadcasts).
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
// topk_read_decode_kernel: the same read for one query row per set, split over a 4-CTA cluster (see below).
#pragma once

#include <cooperative_groups.h>
#include <math_constants.h>

#include "common.cuh"

namespace xencb {

constexpr int SEL_THREADS = 256;
constexpr int SEL_SPT = 4;          // slots per thread
constexpr int SEL_TILE = 32 * SEL_SPT;  // slots per CTA
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

// G: the GQA group size (query heads per KV head); each thread scores SEL_SPT slots (lane + 32 u) of one KV head,
// so every broadcast q load feeds SEL_SPT x 8 FMAs.
template <typename TK, int G>
__global__ void __launch_bounds__(SEL_THREADS) select_scores_kernel(const SelectArgs a) {
  __shared__ float red[SEL_MAX_KV][SEL_TILE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.y;
  const int64_t lib = row / a.rows_per_lib;
  const int S = a.n_chunks * a.page_rows;
  const int base = blockIdx.x * SEL_TILE;
  const int d_k = a.n_kv * a.hd;
  const TK* kb = static_cast<const TK*>(a.keys) + lib * a.keys_lib_stride;
  const float* qrow = a.q + row * (int64_t)a.T * a.n_q * a.hd;

  auto dot8 = [](float sv, const float4& q0, const float4& q1, const float* k) {
    sv = fmaf(q0.x, k[0], sv); sv = fmaf(q0.y, k[1], sv); sv = fmaf(q0.z, k[2], sv); sv = fmaf(q0.w, k[3], sv);
    sv = fmaf(q1.x, k[4], sv); sv = fmaf(q1.y, k[5], sv); sv = fmaf(q1.z, k[6], sv); sv = fmaf(q1.w, k[7], sv);
    return sv;
  };
  auto load_k = [&](const TK* p, float* out) {
    if constexpr (sizeof(TK) == 4) {
      unpack16<float>(__ldg(reinterpret_cast<const uint4*>(p)), out);
      unpack16<float>(__ldg(reinterpret_cast<const uint4*>(p + 4)), out + 4);
    } else {
      unpack16<TK>(__ldg(reinterpret_cast<const uint4*>(p)), out);
    }
  };
  const float init_h = a.h_pool == 0 ? -CUDART_INF_F : 0.f;
  for (int kv = warp; kv < a.n_kv; kv += SEL_THREADS / 32) {
    const TK* kr[SEL_SPT];
#pragma unroll
    for (int u = 0; u < SEL_SPT; ++u) {
      const int slot = base + lane + 32 * u;
      kr[u] = kb + (int64_t)(slot < S ? slot : 0) * d_k + kv * a.hd;  // slots past S read slot 0, never stored
    }
    float p[SEL_SPT];
#pragma unroll
    for (int u = 0; u < SEL_SPT; ++u) p[u] = init_h;
    if (a.T == 1) {
      // one position: the group's heads share every key load
      const float* qk = qrow + (int64_t)kv * G * a.hd;
      if constexpr (sizeof(TK) == 2 && G <= 4) {
        if (a.hd <= 128) {
          // 16-bit keys, head rows of up to 256 bytes: a half-warp reads one slot's head row in one coalesced
          // request (lane l: elements [8 (l & 15), +8) of slot 2 j + (l >> 4)), four slot pairs in flight per
          // lane; the group's q values stay in registers and 16-lane shuffle trees finish the dots
          const int hl = lane & 15, half = lane >> 4;
          const bool el = hl * 8 < a.hd;
          float qv[G][8];
#pragma unroll
          for (int h = 0; h < G; ++h) {
            float4 q0 = make_float4(0.f, 0.f, 0.f, 0.f), q1 = q0;
            if (el) {
              q0 = __ldg(reinterpret_cast<const float4*>(qk + h * a.hd + hl * 8));
              q1 = __ldg(reinterpret_cast<const float4*>(qk + h * a.hd + hl * 8 + 4));
            }
            qv[h][0] = q0.x; qv[h][1] = q0.y; qv[h][2] = q0.z; qv[h][3] = q0.w;
            qv[h][4] = q1.x; qv[h][5] = q1.y; qv[h][6] = q1.z; qv[h][7] = q1.w;
          }
          constexpr int SU = 4;
          for (int sp = 0; sp < SEL_TILE; sp += 2 * SU) {
            uint4 raw[SU];
#pragma unroll
            for (int u = 0; u < SU; ++u) {
              const int slot = base + sp + 2 * u + half;
              const int sl = slot < S ? slot : 0;  // slots past S read slot 0, never stored
              raw[u] = el ? __ldg(reinterpret_cast<const uint4*>(kb + (int64_t)sl * d_k + kv * a.hd + hl * 8))
                          : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < SU; ++u) {
              float kx[8];
              unpack16<TK>(raw[u], kx);
              float pv = init_h;
#pragma unroll
              for (int h = 0; h < G; ++h) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) d = fmaf(qv[h][e], kx[e], d);
                d += __shfl_xor_sync(0xffffffffu, d, 8);
                d += __shfl_xor_sync(0xffffffffu, d, 4);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                pv = a.h_pool == 0 ? fmaxf(pv, d) : pv + d;
              }
              if (hl == 0) red[kv][sp + 2 * u + half] = pv;
            }
          }
          continue;
        }
      }
      float acc[SEL_SPT][G];
#pragma unroll
      for (int u = 0; u < SEL_SPT; ++u)
#pragma unroll
        for (int i = 0; i < G; ++i) acc[u][i] = 0.f;
      for (int e = 0; e < a.hd; e += 8) {
        float kx[SEL_SPT][8];
#pragma unroll
        for (int u = 0; u < SEL_SPT; ++u) load_k(kr[u] + e, kx[u]);
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {  // every lane reads the same q address: a broadcast
          const float4 q0 = __ldg(reinterpret_cast<const float4*>(qk + hh * a.hd + e));
          const float4 q1 = __ldg(reinterpret_cast<const float4*>(qk + hh * a.hd + e + 4));
#pragma unroll
          for (int u = 0; u < SEL_SPT; ++u) acc[u][hh] = dot8(acc[u][hh], q0, q1, kx[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < SEL_SPT; ++u)
#pragma unroll
        for (int hh = 0; hh < G; ++hh) p[u] = a.h_pool == 0 ? fmaxf(p[u], acc[u][hh]) : p[u] + acc[u][hh];
    } else {
      // several positions: per head, pool its scores over the positions (keys re-read from L1 / L2)
      for (int hh = 0; hh < G; ++hh) {
        float hv[SEL_SPT];
#pragma unroll
        for (int u = 0; u < SEL_SPT; ++u) hv[u] = a.t_pool == 0 ? -CUDART_INF_F : 0.f;
        for (int t = 0; t < a.T; ++t) {
          const float* qh = qrow + ((int64_t)t * a.n_q + kv * G + hh) * a.hd;
          float acc[SEL_SPT];
#pragma unroll
          for (int u = 0; u < SEL_SPT; ++u) acc[u] = 0.f;
          for (int e = 0; e < a.hd; e += 8) {
            const float4 q0 = __ldg(reinterpret_cast<const float4*>(qh + e));
            const float4 q1 = __ldg(reinterpret_cast<const float4*>(qh + e + 4));
#pragma unroll
            for (int u = 0; u < SEL_SPT; ++u) {
              float kx[8];
              load_k(kr[u] + e, kx);
              acc[u] = dot8(acc[u], q0, q1, kx);
            }
          }
#pragma unroll
          for (int u = 0; u < SEL_SPT; ++u) hv[u] = a.t_pool == 0 ? fmaxf(hv[u], acc[u]) : hv[u] + acc[u];
        }
#pragma unroll
        for (int u = 0; u < SEL_SPT; ++u) {
          const float v = a.t_pool == 0 ? hv[u] : hv[u] / (float)a.T;
          p[u] = a.h_pool == 0 ? fmaxf(p[u], v) : p[u] + v;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < SEL_SPT; ++u) red[kv][lane + 32 * u] = p[u];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < SEL_TILE; j += SEL_THREADS) {
    const int slot = base + j;
    if (slot >= S) continue;
    float p = a.h_pool == 0 ? -CUDART_INF_F : 0.f;
    for (int kv = 0; kv < a.n_kv; ++kv) {
      const float v = red[kv][j];
      p = a.h_pool == 0 ? fmaxf(p, v) : p + v;
    }
    if (a.h_pool == 1) p /= (float)a.n_q;
    const int c = slot / a.page_rows, n = slot - c * a.page_rows;
    const int nc = a.n_chunks_of ? a.n_chunks_of[lib] : a.n_chunks;
    const bool valid = c < nc && n < a.n_valid[lib * a.n_chunks + c];
    a.scores[row * (int64_t)S + slot] = valid ? p : -CUDART_INF_F;
  }
}

// One query position, f16 keys, GQA groups G <= 4, head rows of 32 P2 elements (P2 = 1, 2, 4): the dot
// products on the tensor cores. Per KV head, an m16n8k16 chain scores 16 slots (MMA rows) against 8 columns: the
// group's G query heads rounded to f16 (hi) and their remainders q - hi (lo), both after a power-of-two scale per
// (row, KV head) that puts max|q| in [2^13, 2^14); the score of head h is (D[:, h] + D[:, G + h]) / scale. The keys
// are exact in f16 and the products exact in the f32 accumulator, so the error is that of a ~22-bit q (the same
// 1e-5 bar as the f32 path). The A fragments are loaded from global memory directly: lane (g, t) reads 16 bytes
// of slot rows g and g + 8 at element 32 j + 8 t of the head row, so four lanes cover 64 contiguous bytes of a
// row; this assigns the contraction index of k-step 2 j + e as  kk -> 32 j + 8 (kk % 8 / 2) + 4 e + 2 (kk / 8)
// + kk % 2, and the B fragments (q) follow the same map. Warp w takes KV heads w, w + 8, ... over the CTA's
// SEL_TILE slots, two 16-slot groups of loads in flight; the per-head pooling goes through a 16 x 8 shared tile
// per warp, the pooling over KV heads and the validity as in select_scores_kernel.
constexpr int SELM_GROUPS = SEL_TILE / 16;

template <int G, int P2>
__global__ void __launch_bounds__(SEL_THREADS, 2) select_scores_mma_kernel(const SelectArgs a) {
  __shared__ float red[SEL_MAX_KV][SEL_TILE];
  __shared__ float dt[SEL_THREADS / 32][16][9];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t row = blockIdx.y;
  const int64_t lib = row / a.rows_per_lib;
  const int S = a.n_chunks * a.page_rows;
  const int base = blockIdx.x * SEL_TILE;
  const int hd = 32 * P2;
  const int d_k = a.n_kv * hd;
  const __half* kb = static_cast<const __half*>(a.keys) + lib * a.keys_lib_stride;
  const float* qrow = a.q + row * (int64_t)a.n_q * hd;
  const float init_h = a.h_pool == 0 ? -CUDART_INF_F : 0.f;
  float (*tile)[9] = dt[warp];
  for (int kv = warp; kv < a.n_kv; kv += SEL_THREADS / 32) {
    const float* qk = qrow + (int64_t)kv * G * hd;
    uint4 ra[2][P2], rb[2][P2];
    auto load = [&](int gi) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        int s0 = base + 16 * (gi + u) + g, s1 = s0 + 8;
        s0 = s0 < S ? s0 : S - 1;  // slots past S read the last slot, never stored
        s1 = s1 < S ? s1 : S - 1;
        const __half* p0 = kb + (int64_t)s0 * d_k + kv * hd + 8 * t;
        const __half* p1 = kb + (int64_t)s1 * d_k + kv * hd + 8 * t;
#pragma unroll
        for (int j = 0; j < P2; ++j) {
          ra[u][j] = __ldg(reinterpret_cast<const uint4*>(p0 + 32 * j));
          rb[u][j] = __ldg(reinterpret_cast<const uint4*>(p1 + 32 * j));
        }
      }
    };
    load(0);  // the first keys are in flight while q is prepared
    // scale: a power of two that puts the group's max|q| in [2^13, 2^14)
    float mx = 0.f;
    for (int i = lane; i < G * hd; i += 32) mx = fmaxf(mx, fabsf(__ldg(qk + i)));
    mx = warp_max(mx);
    int ex = 0;
    if (mx > 0.f && mx <= 3.0e38f) frexpf(mx, &ex);
    const float sc = (mx > 0.f && mx <= 3.0e38f) ? ldexpf(1.f, 14 - ex) : 1.f;
    const float inv = 1.f / sc;  // exact: a power of two
    // B fragments: column g is hi of head g (g < G), lo of head g - G (G <= g < 2 G), else 0
    uint32_t bq[4 * P2][2];
#pragma unroll
    for (int ks = 0; ks < 4 * P2; ++ks) {
      const int e0 = 32 * (ks >> 1) + 8 * t + 4 * (ks & 1);
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (g < 2 * G) {
        const float* qh = qk + (g % G) * hd + e0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float x = __ldg(qh + i) * sc;
          const float hi = __half2float(__float2half_rn(x));
          v[i] = g < G ? hi : x - hi;
        }
      }
      float r0, r1;
      bq[ks][0] = pack2<__half>(v[0], v[1], r0, r1);
      bq[ks][1] = pack2<__half>(v[2], v[3], r0, r1);
    }
    for (int gi = 0; gi < SELM_GROUPS; gi += 2) {
      if (gi) load(gi);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < P2; ++j) {
          mma16816<__half>(d, ra[u][j].x, rb[u][j].x, ra[u][j].y, rb[u][j].y, bq[2 * j][0], bq[2 * j][1]);
          mma16816<__half>(d, ra[u][j].z, rb[u][j].z, ra[u][j].w, rb[u][j].w, bq[2 * j + 1][0], bq[2 * j + 1][1]);
        }
        tile[g][2 * t] = d[0];
        tile[g][2 * t + 1] = d[1];
        tile[g + 8][2 * t] = d[2];
        tile[g + 8][2 * t + 1] = d[3];
        __syncwarp();
        if (lane < 16) {
          float pv = init_h;
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float x = (tile[lane][h] + tile[lane][G + h]) * inv;
            pv = a.h_pool == 0 ? fmaxf(pv, x) : pv + x;
          }
          red[kv][16 * (gi + u) + lane] = pv;
        }
        __syncwarp();
      }
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < SEL_TILE; j += SEL_THREADS) {
    const int slot = base + j;
    if (slot >= S) continue;
    float p = init_h;
    for (int kv = 0; kv < a.n_kv; ++kv) {
      const float v = red[kv][j];
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

// The same selection for rows of up to TKC_CL * TKC_THREADS * TKC_KPT slots, spread over a cluster of TKC_CL
// CTAs: CTA c owns the contiguous slots [c * slice, (c + 1) * slice), held in registers (thread t: TKC_KPT
// consecutive slots). Each radix pass builds the CTA's histogram (per-warp packed histograms as above), and after
// one cluster barrier every CTA sums the TKC_CL histograms through distributed shared memory and takes the same
// bin (histograms alternate between two buffers by pass, so a CTA never overwrites one another CTA may still
// read). The compaction scans the CTAs' (greater, equal) counts in cluster order, which is slot order, so ties at
// the threshold still go to the lower slots; each CTA writes its winners into CTA 0's arrays, which sorts them.
// Per-warp histograms (two 16-bit bins per word, at most 32 * TKC_KPT per bin) keep the first pass, where nearly
// every key falls in one or two bins, from serialising the CTA on those bins' atomics.
constexpr int TKC_CL = 8;
constexpr int TKC_THREADS = 512;
constexpr int TKC_KPT = 8;

__global__ void __cluster_dims__(TKC_CL, 1, 1) __launch_bounds__(TKC_THREADS)
    select_topk_cluster_kernel(const float* __restrict__ scores, int S, int k, int32_t* __restrict__ idx_out,
                               float* __restrict__ score_out) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ uint32_t whist[TKC_THREADS / 32][128];
  __shared__ int hist[2][256];
  __shared__ int tot[256];
  __shared__ int sh_bin, sh_rem;
  __shared__ int cnt_gt[TKC_THREADS], cnt_eq[TKC_THREADS];
  __shared__ int cta_cnt[2];
  __shared__ uint32_t skey[TOPK_MAX_K];
  __shared__ int sidx[TOPK_MAX_K];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int crank = (int)cluster.block_rank();
  const int64_t row = blockIdx.x / TKC_CL;
  const float* sc = scores + row * S;
  const int slice = (S + TKC_CL - 1) / TKC_CL;
  const int i0 = crank * slice + tid * TKC_KPT;
  const int iend = min(S, (crank + 1) * slice);
  uint32_t key[TKC_KPT];
#pragma unroll
  for (int j = 0; j < TKC_KPT; ++j) key[j] = i0 + j < iend ? order_key(__ldg(sc + i0 + j)) : 0u;

  uint32_t prefix = 0, pmask = 0;
  int rem = k;
  int buf = 0;
  for (int shift = 24; shift >= 0; shift -= 8, buf ^= 1) {
    for (int i = lane; i < 128; i += 32) whist[warp][i] = 0u;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < TKC_KPT; ++j) {
      if ((key[j] & pmask) == prefix) {
        const uint32_t b = (key[j] >> shift) & 255u;
        atomicAdd(&whist[warp][b >> 1], 1u << ((b & 1u) << 4));
      }
    }
    __syncthreads();
    if (tid < 256) {
      int t = 0;
      for (int w = 0; w < TKC_THREADS / 32; ++w) t += (int)((whist[w][tid >> 1] >> ((tid & 1) << 4)) & 0xffffu);
      hist[buf][tid] = t;
    }
    cluster.sync();  // every CTA's histogram of this pass is complete
    if (tid < 256) {
      int t = 0;
      for (int r = 0; r < TKC_CL; ++r) t += cluster.map_shared_rank(&hist[buf][0], r)[tid];
      tot[tid] = t;
    }
    __syncthreads();
    if (tid < 32) {
      int part = 0;
      for (int b = 0; b < 8; ++b) part += tot[255 - 8 * tid - b];
      int incl = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += v;
      }
      const int excl = incl - part;
      if (excl < rem && incl >= rem) {
        int run = excl;
        for (int b = 0; b < 8; ++b) {
          const int bin = 255 - 8 * tid - b;
          if (run + tot[bin] >= rem) { sh_bin = bin; sh_rem = rem - run; break; }
          run += tot[bin];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sh_bin << shift;
    pmask |= 255u << shift;
    rem = sh_rem;
  }
  const uint32_t thr = prefix;
  const int take_eq = rem;

  // ---- compaction: thread order within the CTA, CTA order within the cluster (both slot order)
  int ngt = 0, neq = 0;
#pragma unroll
  for (int j = 0; j < TKC_KPT; ++j) {
    ngt += key[j] > thr;
    neq += key[j] == thr;
  }
  cnt_gt[tid] = ngt;
  cnt_eq[tid] = neq;
  __syncthreads();
  for (int o = 1; o < TKC_THREADS; o <<= 1) {
    const int a_gt = tid >= o ? cnt_gt[tid - o] : 0;
    const int a_eq = tid >= o ? cnt_eq[tid - o] : 0;
    __syncthreads();
    cnt_gt[tid] += a_gt;
    cnt_eq[tid] += a_eq;
    __syncthreads();
  }
  if (tid == 0) {
    cta_cnt[0] = cnt_gt[TKC_THREADS - 1];
    cta_cnt[1] = cnt_eq[TKC_THREADS - 1];
  }
  cluster.sync();  // every CTA's totals are published
  int off_gt = 0, off_eq = 0, n_gt_total = 0;
  for (int r = 0; r < TKC_CL; ++r) {
    const int* cc = cluster.map_shared_rank(cta_cnt, r);
    const int g = cc[0], e = cc[1];
    if (r < crank) { off_gt += g; off_eq += e; }
    n_gt_total += g;
  }
  uint32_t* lkey = cluster.map_shared_rank(skey, 0);
  int* lidx = cluster.map_shared_rank(sidx, 0);
  int pos_gt = off_gt + cnt_gt[tid] - ngt, pos_eq = off_eq + cnt_eq[tid] - neq;
#pragma unroll
  for (int j = 0; j < TKC_KPT; ++j) {
    if (key[j] > thr) {
      lkey[pos_gt] = key[j]; lidx[pos_gt] = i0 + j; ++pos_gt;
    } else if (key[j] == thr) {
      if (pos_eq < take_eq) { lkey[n_gt_total + pos_eq] = key[j]; lidx[n_gt_total + pos_eq] = i0 + j; }
      ++pos_eq;
    }
  }
  cluster.sync();  // CTA 0 holds the k winners; the other CTAs are done
  if (crank != 0) return;
  int kp = 1;
  while (kp < k) kp <<= 1;
  for (int i = k + tid; i < kp; i += TKC_THREADS) { skey[i] = 0u; sidx[i] = 0x7fffffff; }
  __syncthreads();
  for (int size = 2; size <= kp; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < kp; i += TKC_THREADS) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
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
  for (int i = tid; i < k; i += TKC_THREADS) {
    idx_out[row * k + i] = sidx[i];
    if (score_out) score_out[row * k + i] = sc[sidx[i]];
  }
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
__device__ __forceinline__ void load_row8(const char* base, int j, float* out) {
  const T* p = reinterpret_cast<const T*>(base) + j;
  if constexpr (sizeof(T) == 4) {
    unpack16<float>(__ldg(reinterpret_cast<const uint4*>(p)), out);
    unpack16<float>(__ldg(reinterpret_cast<const uint4*>(p + 4)), out + 4);
  } else {
    unpack16<T>(__ldg(reinterpret_cast<const uint4*>(p)), out);
  }
}

// NT: query rows per CTA (1 for decode, TR_ROWS otherwise), so decode does no work for absent rows.
template <typename T, int NT>
__global__ void __launch_bounds__(TR_THREADS) topk_read_kernel(const TopkReadArgs a) {
  extern __shared__ __align__(16) float tr_smem[];
  float* qs = tr_smem;                                   // [NT][d_s]
  float* at = tr_smem + (size_t)NT * a.d_s;              // [NT][k]
  int64_t* koff = reinterpret_cast<int64_t*>(at + (((size_t)NT * a.k + 1) & ~(size_t)1));  // [k] row byte offsets
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int set = blockIdx.x;
  const int64_t t0 = (int64_t)blockIdx.y * NT;
  const int64_t left = a.rows_per_set - t0;
  const int nt = left < NT ? (int)left : NT;
  if (nt <= 0) return;
  const int64_t row0 = (int64_t)set * a.rows_per_set + t0;
  const int64_t lib = a.n_lib > 1 ? set : 0;
  const int32_t* ix = a.idx + (int64_t)set * a.k;
  const int d_s = a.d_s;
  constexpr int ES = (int)sizeof(T);

  // slot -> byte offset of its row in the pool (-1: outside the grid or the pool: scores -inf, reads nothing)
  for (int i = threadIdx.x; i < a.k; i += TR_THREADS) {
    const int s = ix[i];
    int64_t off = -1;
    if (s >= 0 && s < a.n_chunks * a.page_rows) {
      const int c = s / a.page_rows, n = s - c * a.page_rows;
      const int64_t page = a.page_of[lib * a.n_chunks + c];
      if (page >= 0 && page < a.n_pages) off = page * a.page_stride_bytes + (int64_t)n * d_s * ES;
    }
    koff[i] = off;
  }
  for (int j = threadIdx.x * 4; j < NT * d_s; j += TR_THREADS * 4) {
    const int t = j / d_s;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < nt) v = *reinterpret_cast<const float4*>(a.q + (row0 + t) * d_s + (j - t * d_s));
    *reinterpret_cast<float4*>(qs + j) = v;
  }
  __syncthreads();

  // ---- scores: a warp per selected row, the row's 16-byte pieces loaded four at a time
  for (int i = warp; i < a.k; i += TR_THREADS / 32) {
    const int64_t off = koff[i];
    float dot[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) dot[t] = 0.f;
    if (off >= 0) {
      const char* kr = a.slots + off;
#pragma unroll 4
      for (int j = lane * 8; j < d_s; j += 256) {
        float kx[8];
        load_row8<T>(kr, j, kx);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float4 q0 = *reinterpret_cast<const float4*>(qs + t * d_s + j);
          const float4 q1 = *reinterpret_cast<const float4*>(qs + t * d_s + j + 4);
          float sv = dot[t];
          sv = fmaf(q0.x, kx[0], sv); sv = fmaf(q0.y, kx[1], sv); sv = fmaf(q0.z, kx[2], sv); sv = fmaf(q0.w, kx[3], sv);
          sv = fmaf(q1.x, kx[4], sv); sv = fmaf(q1.y, kx[5], sv); sv = fmaf(q1.z, kx[6], sv); sv = fmaf(q1.w, kx[7], sv);
          dot[t] = sv;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float sv = warp_sum(dot[t]);
      if (lane == 0) at[t * a.k + i] = off >= 0 ? sv : -CUDART_INF_F;
    }
  }
  __syncthreads();
  // ---- per query row: softmax over the k scores (or the linear 1/sqrt(k) scale)
  for (int t = warp; t < nt; t += TR_THREADS / 32) {
    float* ar = at + t * a.k;
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
      for (int i = lane; i < a.k; i += 32) a.attn_out[(row0 + t) * a.k + i] = ar[i];
  }
  __syncthreads();
  // ---- r = a @ V over the selected rows: a thread owns 8 columns; four value rows in flight per step
  const char* vpool = a.vslots ? a.vslots : a.slots;
  for (int j = threadIdx.x * 8; j < d_s; j += TR_THREADS * 8) {
    float acc[NT][8];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[t][e] = 0.f;
    for (int i0 = 0; i0 < a.k; i0 += 4) {
      float vx[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u;
        const int64_t off = i < a.k ? koff[i] : -1;
        if (off >= 0) load_row8<T>(vpool + off, j, vx[u]);
        else {
#pragma unroll
          for (int e = 0; e < 8; ++e) vx[u][e] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u;
        if (i >= a.k) break;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float w = at[t * a.k + i];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[t][e] = fmaf(w, vx[u][e], acc[t][e]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < nt) {
        float* o = a.r_out + (row0 + t) * d_s + j;
        *reinterpret_cast<float4*>(o) = make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(acc[t][4], acc[t][5], acc[t][6], acc[t][7]);
      }
    }
  }
}

// Decode form (one query row per index set): a cluster of TRC CTAs per set splits the k selected rows; the
// softmax maximum and sum and the partial weighted sums are combined through distributed shared memory, so a
// document's rows stream through TRC SMs at once. CTA `rank` writes columns [rank, rank + TRC, ...) in 8-column
// groups of the combined r.
constexpr int TRC = 4;

template <typename T>
__global__ void __cluster_dims__(TRC, 1, 1) __launch_bounds__(TR_THREADS)
topk_read_decode_kernel(const TopkReadArgs a) {
  extern __shared__ __align__(16) float trd_smem[];
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int d_s = a.d_s;
  const int per = (a.k + TRC - 1) / TRC;                 // rows per CTA
  const int i0 = min(a.k, rank * per), i1 = min(a.k, i0 + per), nl = i1 - i0;
  float* qs = trd_smem;                                  // [d_s]
  float* part = qs + d_s;                                // [d_s] this CTA's partial r
  float* at = part + d_s;                                // [per] scores -> weights
  float* stats = at + ((per + 3) & ~3);                  // [4]: local max, local sum
  int64_t* koff = reinterpret_cast<int64_t*>(stats + 4); // [per]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int set = blockIdx.x / TRC;
  const int64_t row = set;  // one query row per set
  const int64_t lib = a.n_lib > 1 ? set : 0;
  const int32_t* ix = a.idx + (int64_t)set * a.k;
  constexpr int ES = (int)sizeof(T);

  for (int i = threadIdx.x; i < nl; i += TR_THREADS) {
    const int s = ix[i0 + i];
    int64_t off = -1;
    if (s >= 0 && s < a.n_chunks * a.page_rows) {
      const int c = s / a.page_rows, n = s - c * a.page_rows;
      const int64_t page = a.page_of[lib * a.n_chunks + c];
      if (page >= 0 && page < a.n_pages) off = page * a.page_stride_bytes + (int64_t)n * d_s * ES;
    }
    koff[i] = off;
  }
  for (int j = threadIdx.x * 4; j < d_s; j += TR_THREADS * 4)
    *reinterpret_cast<float4*>(qs + j) = *reinterpret_cast<const float4*>(a.q + row * d_s + j);
  __syncthreads();

  // ---- scores of this CTA's rows: a warp per row, the row's pieces loaded eight at a time
  for (int i = warp; i < nl; i += TR_THREADS / 32) {
    const int64_t off = koff[i];
    float dot = 0.f;
    if (off >= 0) {
      const char* kr = a.slots + off;
#pragma unroll 8
      for (int j = lane * 8; j < d_s; j += 256) {
        float kx[8];
        load_row8<T>(kr, j, kx);
        const float4 q0 = *reinterpret_cast<const float4*>(qs + j);
        const float4 q1 = *reinterpret_cast<const float4*>(qs + j + 4);
        dot = fmaf(q0.x, kx[0], dot); dot = fmaf(q0.y, kx[1], dot); dot = fmaf(q0.z, kx[2], dot);
        dot = fmaf(q0.w, kx[3], dot); dot = fmaf(q1.x, kx[4], dot); dot = fmaf(q1.y, kx[5], dot);
        dot = fmaf(q1.z, kx[6], dot); dot = fmaf(q1.w, kx[7], dot);
      }
    }
    dot = warp_sum(dot);
    if (lane == 0) at[i] = off >= 0 ? dot : -CUDART_INF_F;
  }
  __syncthreads();
  // ---- softmax statistics across the cluster (warp 0 of each CTA)
  if (a.softmax) {
    if (warp == 0) {
      float mx = -CUDART_INF_F;
      for (int i = lane; i < nl; i += 32) mx = fmaxf(mx, at[i] * a.qscale);
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) stats[0] = mx;
    }
    cluster.sync();
    float gmax = -CUDART_INF_F;
    for (int r = 0; r < TRC; ++r) gmax = fmaxf(gmax, *cluster.map_shared_rank(stats, r));
    if (warp == 0) {
      float sum = 0.f;
      for (int i = lane; i < nl; i += 32) {
        const float e = at[i] == -CUDART_INF_F ? 0.f : exp2f(at[i] * a.qscale - gmax);
        at[i] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) stats[1] = sum;
    }
    cluster.sync();
    float gsum = 0.f;
    for (int r = 0; r < TRC; ++r) gsum += *cluster.map_shared_rank(stats + 1, r);
    const float inv = 1.f / gsum;
    for (int i = threadIdx.x; i < nl; i += TR_THREADS) at[i] *= inv;
  } else {
    const float sc = rsqrtf((float)a.k);
    for (int i = threadIdx.x; i < nl; i += TR_THREADS) at[i] = at[i] == -CUDART_INF_F ? 0.f : at[i] * sc;
  }
  __syncthreads();
  if (a.attn_out)
    for (int i = threadIdx.x; i < nl; i += TR_THREADS) a.attn_out[row * a.k + i0 + i] = at[i];
  // ---- this CTA's partial r over its rows: a thread owns 8 columns, eight value rows in flight per step
  const char* vpool = a.vslots ? a.vslots : a.slots;
  for (int j = threadIdx.x * 8; j < d_s; j += TR_THREADS * 8) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int b = 0; b < nl; b += 8) {
      float vx[8][8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t off = b + u < nl ? koff[b + u] : -1;
        if (off >= 0) load_row8<T>(vpool + off, j, vx[u]);
        else {
#pragma unroll
          for (int e = 0; e < 8; ++e) vx[u][e] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = b + u < nl ? at[b + u] : 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(w, vx[u][e], acc[e]);
      }
    }
    *reinterpret_cast<float4*>(part + j) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(part + j + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  cluster.sync();
  // ---- combine the partials: this CTA sums the 8-column groups g = rank, rank + TRC, ... over the cluster
  for (int g8 = rank + TRC * (int)threadIdx.x; g8 * 8 < d_s; g8 += TRC * TR_THREADS) {
    const int j = g8 * 8;
    float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
    for (int r = 0; r < TRC; ++r) {
      const float* pr = cluster.map_shared_rank(part, r) + j;
      const float4 x0 = *reinterpret_cast<const float4*>(pr), x1 = *reinterpret_cast<const float4*>(pr + 4);
      s0.x += x0.x; s0.y += x0.y; s0.z += x0.z; s0.w += x0.w;
      s1.x += x1.x; s1.y += x1.y; s1.z += x1.z; s1.w += x1.w;
    }
    float* o = a.r_out + row * d_s + j;
    *reinterpret_cast<float4*>(o) = s0;
    *reinterpret_cast<float4*>(o + 4) = s1;
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
}

}  // namespace xencb

// Decode read over routed chunks: the hot op of LibraryInjector._branch (xenc/injector.py:239-245, 263-265)
// for query rows that each read their own top-k chunks.
//
// Work items. Item (row, j, s) reads rows [s*split_rows, min(n_valid, (s+1)*split_rows)) of chunk
// c = idx[row, j] and produces a partial (m, l, acc[d_s]) of the chunk softmax (log2 domain):
//     m = max_n s_n, l = sum_n 2^(s_n - m), acc = sum_n 2^(s_n - m) k_n,  s_n = (read_temp*log2 e) q . k_n
// Because K = V (tied), each slot row is fetched from HBM exactly once and used for both the score and the
// accumulation. read_merge_kernel combines the splits of a chunk by log-sum-exp and the chunks by the
// routing weights.
//
// CTA shape (persistent, one per SM): warp 0 lane 0 is the producer -- it walks the CTA's items and issues
// one 1-D cp.async.bulk (TMA, no multicast) per stage of `rps` consecutive slot rows into a ring of
// `n_stage` shared-memory stages, each guarded by a full/empty mbarrier pair. Warps 1..ncw are consumers:
// consumer thread t owns the 16-byte column vectors t + i*32*ncw (i < VPT) of every row, so a warp's
// shared-memory reads are 512 contiguous bytes. Rows are scored in groups of 8: each thread forms 8 partial
// dot products, a transposed butterfly leaves each lane with one row's warp total (9 shuffles), warps meet
// in a double-buffered shared array behind one named barrier, and lane i of every warp finishes row i & 7,
// takes the exp2 and broadcasts the 8 weights. The online softmax state (m, l) is uniform across the CTA.
//
// Every mbarrier wait is bounded (XENCB_WAIT_CYCLES); a consumer that gives up raises a shared abort flag that
// all consumers test after the next named barrier (or warp vote), so no thread is left at a barrier.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace xencb {

constexpr int RD_G = 8;  // rows per scoring group

struct ReadArgs {
  const float* q;
  int64_t n_rows;
  int d_s;
  const char* slots;
  const char* vslots;  // untied values (same page layout as slots), or null when V = K
  int64_t n_pages;
  int64_t page_stride_bytes;
  int page_rows;
  const int32_t* page_of;
  const int32_t* n_valid;
  int n_chunks;
  int64_t rows_per_lib;
  const int32_t* idx;
  const float* wk;
  int k;
  float qscale;  // read_temp * log2(e) for the softmax read, 1 for the linear read
  int n_split, split_rows, rps, n_stage, row_bytes, nvec;
  int row_stride;  // shared-memory bytes between staged rows (the tensor-core kernel pads rows by 16 B)
  int64_t n_items;
  float* part_acc;  // [n_items, d_s]
  float* part_ml;   // [n_items, 2]
  // sparse plan (xencb_read_decode_sparse): the items that hold rows, in item order, and their count, written by
  // read_compact_kernel; null for the dense plan, whose CTAs walk every item
  const int32_t* item_list;
  const int* n_active;
  // the same plan built inside the tensor-core read kernel (no list, no extra launch): for up to RM_PLAN_PAIRS
  // pairs every CTA counts the live pieces of each pair and scans them in shared memory; 0 = off
  int plan_pairs;
};

constexpr int RM_PLAN_PAIRS = 1024;

// Pieces of pair `pr` that hold rows (routed chunk valid, weight != 0, page in the pool): the read_compact count.
__device__ __forceinline__ int pair_pieces(const ReadArgs& a, int64_t pr) {
  const int32_t c = a.idx[pr];
  const float w = a.wk[pr];
  if (c < 0 || c >= a.n_chunks || w == 0.f) return 0;
  const int64_t lc = (pr / a.k / a.rows_per_lib) * a.n_chunks + c;
  const int64_t page = a.page_of[lc];
  if (page < 0 || page >= a.n_pages) return 0;  // decode_item flags it
  int nv = a.n_valid[lc];
  if (nv > a.page_rows) nv = a.page_rows;
  if (nv < 0) nv = 0;
  return min(a.n_split, (nv + a.split_rows - 1) / a.split_rows);
}

struct ItemRange {
  int64_t row;
  int r0, r1;  // slot rows [r0, r1) of the chunk
  const char* base;  // page base
  bool active;       // weight > 0 and a valid chunk id
};

__device__ __forceinline__ ItemRange decode_item(const ReadArgs& a, int64_t item) {
  ItemRange it;
  const int64_t pair = item / a.n_split;
  const int s = (int)(item - pair * a.n_split);
  it.row = pair / a.k;
  const int32_t c = a.idx[pair];
  const float w = a.wk[pair];
  it.active = (c >= 0) && (c < a.n_chunks) && (w != 0.f);
  it.r0 = 0; it.r1 = 0; it.base = nullptr;
  if (!it.active) return it;
  const int64_t lib = it.row / a.rows_per_lib;
  const int64_t lc = lib * a.n_chunks + c;
  const int64_t page = a.page_of[lc];
  if (page < 0 || page >= a.n_pages) {  // never read outside the pool
    if (s == 0) flag_error(XENCB_DEV_BADPAGE);
    it.active = false;
    return it;
  }
  int nv = a.n_valid[lc];
  if (nv > a.page_rows) { nv = a.page_rows; flag_error(XENCB_DEV_CLAMPED); }
  if (nv < 0) nv = 0;
  it.r0 = s * a.split_rows;
  it.r1 = min(nv, it.r0 + a.split_rows);
  if (it.r1 < it.r0) it.r1 = it.r0;
  it.base = a.slots + page * a.page_stride_bytes;
  return it;
}

template <typename T, int VPT, bool SOFTMAX>
__global__ void __launch_bounds__(512, 1) read_decode_kernel(const ReadArgs a) {
  constexpr int EPV = Vec16<T>::n;  // elements per 16-byte vector
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = (blockDim.x >> 5) - 1;
  const int stage_bytes = ((a.rps * a.row_bytes + 127) / 128) * 128;
  unsigned char* stages = smem;
  float* red = reinterpret_cast<float*>(smem + (size_t)a.n_stage * stage_bytes);  // [2][ncw][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * ncw * RD_G);
  uint64_t* empty = full + a.n_stage;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + a.n_stage);

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.n_stage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], ncw);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // ------------------------------------------------------------------------------------------- producer
  if (warp == 0) {
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    uint32_t it_count = 0;  // stages issued so far
    bool ok = true;
    for (int64_t item = blockIdx.x; item < a.n_items && ok; item += gridDim.x) {
      const ItemRange it = decode_item(a, item);
      if (!it.active) continue;
      for (int rs = it.r0; rs < it.r1; rs += a.rps) {
        const int nr = min(a.rps, it.r1 - rs);
        const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
        if (use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) { ok = false; break; }
        const uint32_t bytes = (uint32_t)nr * a.row_bytes;
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(stages + (size_t)slot * stage_bytes, it.base + (int64_t)rs * a.row_bytes, bytes, &full[slot], pol);
        ++it_count;
      }
    }
    // drain: the most recent copy into each stage has landed before the CTA may exit
    const uint32_t n_slots = it_count < (uint32_t)a.n_stage ? it_count : (uint32_t)a.n_stage;
    for (uint32_t i = 0; i < n_slots; ++i) {
      const uint32_t last = it_count - 1 - i;
      mbar_wait_bounded(&full[last % a.n_stage], (last / a.n_stage) & 1);
    }
    return;
  }

  // ------------------------------------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int ct = threadIdx.x - 32;
  const int nct = ncw * 32;
  bool vok[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) vok[i] = (i * nct + ct) < a.nvec;

  uint32_t it_count = 0;
  uint32_t grp = 0;  // scoring groups processed (red buffer parity)
  bool aborted = false;

  for (int64_t item = blockIdx.x; item < a.n_items && !aborted; item += gridDim.x) {
    const ItemRange it = decode_item(a, item);
    if (!it.active) continue;

    float qf[VPT][EPV];
    const float* qr = a.q + it.row * a.d_s;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = i * nct + ct;
#pragma unroll
      for (int e = 0; e < EPV; ++e) qf[i][e] = vok[i] ? __ldg(qr + v * EPV + e) * a.qscale : 0.f;
    }
    float acc[VPT][EPV];
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[i][e] = 0.f;
    float m = -CUDART_INF_F, l = 0.f;

    for (int rs = it.r0; rs < it.r1 && !aborted; rs += a.rps) {
      const int nr = min(a.rps, it.r1 - rs);
      const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
      ++it_count;
      if (!mbar_wait_bounded(&full[slot], use & 1)) *abort_flag = 1;
      const unsigned char* st = stages + (size_t)slot * stage_bytes;

      for (int g0 = 0; g0 < nr; g0 += RD_G) {
        const int gv = min(RD_G, nr - g0);
        // VPT == 1 keeps the group's rows in registers between the score and the accumulation;
        // VPT == 2 reads them from shared memory a second time instead (register budget).
        constexpr bool KEEP = VPT == 1;
        uint4 kr[KEEP ? RD_G : 1][VPT];
        float part[RD_G];
#pragma unroll
        for (int r = 0; r < RD_G; ++r) {
          part[r] = 0.f;
#pragma unroll
          for (int i = 0; i < VPT; ++i) {
            uint4 raw = make_uint4(0u, 0u, 0u, 0u);
            if (r < gv && vok[i])
              raw = *reinterpret_cast<const uint4*>(st + (size_t)(g0 + r) * a.row_bytes + (size_t)(i * nct + ct) * 16);
            if (KEEP) kr[KEEP ? r : 0][i] = raw;
            float kf[EPV];
            unpack16<T>(raw, kf);
#pragma unroll
            for (int e = 0; e < EPV; ++e) part[r] = fmaf(qf[i][e], kf[e], part[r]);
          }
        }
        // transposed butterfly: lane ends with the warp total of row (lane >> 2)
        {
          const bool b16 = lane & 16;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float send = b16 ? part[i] : part[i + 4];
            const float keep = b16 ? part[i + 4] : part[i];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
          }
          const bool b8 = lane & 8;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float send = b8 ? part[i] : part[i + 2];
            const float keep = b8 ? part[i + 2] : part[i];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
          }
          const bool b4 = lane & 4;
          {
            const float send = b4 ? part[0] : part[1];
            const float keep = b4 ? part[1] : part[0];
            part[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
          }
          part[0] += __shfl_xor_sync(0xffffffffu, part[0], 2);
          part[0] += __shfl_xor_sync(0xffffffffu, part[0], 1);
        }
        // lane -> score of row (lane & 7)
        float srow;
        if (ncw > 1) {
          float* rb = red + (grp & 1) * ncw * RD_G;
          if ((lane & 3) == 0) rb[cw * RD_G + (lane >> 2)] = part[0];
          named_bar_sync(1, nct);
          if (*abort_flag) { aborted = true; break; }
          srow = 0.f;
          for (int w = 0; w < ncw; ++w) srow += rb[w * RD_G + (lane & 7)];
        } else {
          if (__any_sync(0xffffffffu, *abort_flag != 0)) { aborted = true; break; }
          srow = __shfl_sync(0xffffffffu, part[0], (lane & 7) * 4);
        }
        ++grp;
        const bool valid = (lane & 7) < gv;
        float pw[RD_G];
        if (SOFTMAX) {
          float mx = valid ? srow : -CUDART_INF_F;
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          const float m_new = fmaxf(m, mx);
          if (m_new != m) {
            const float sc = exp2f(m - m_new);
            l *= sc;
#pragma unroll
            for (int i = 0; i < VPT; ++i)
#pragma unroll
              for (int e = 0; e < EPV; ++e) acc[i][e] *= sc;
            m = m_new;
          }
          const float p = valid ? exp2f(srow - m) : 0.f;
          float ps = p;
          ps += __shfl_xor_sync(0xffffffffu, ps, 1);
          ps += __shfl_xor_sync(0xffffffffu, ps, 2);
          ps += __shfl_xor_sync(0xffffffffu, ps, 4);
          l += ps;
#pragma unroll
          for (int r = 0; r < RD_G; ++r) pw[r] = __shfl_sync(0xffffffffu, p, r);
        } else {
          const float p = valid ? srow : 0.f;
#pragma unroll
          for (int r = 0; r < RD_G; ++r) pw[r] = __shfl_sync(0xffffffffu, p, r);
        }
#pragma unroll
        for (int r = 0; r < RD_G; ++r) {
#pragma unroll
          for (int i = 0; i < VPT; ++i) {
            uint4 raw;
            if (KEEP) {
              raw = kr[KEEP ? r : 0][i];
            } else {
              raw = make_uint4(0u, 0u, 0u, 0u);
              if (r < gv && vok[i])
                raw = *reinterpret_cast<const uint4*>(st + (size_t)(g0 + r) * a.row_bytes + (size_t)(i * nct + ct) * 16);
            }
            float kf[EPV];
            unpack16<T>(raw, kf);
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[i][e] = fmaf(pw[r], kf[e], acc[i][e]);
          }
        }
      }
      // release the stage
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (aborted) break;

    // partial out
    float* pa = a.part_acc + item * (int64_t)a.d_s;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (!vok[i]) continue;
      const int v = i * nct + ct;
#pragma unroll
      for (int e = 0; e < EPV; e += 4)
        *reinterpret_cast<float4*>(pa + v * EPV + e) = make_float4(acc[i][e], acc[i][e + 1], acc[i][e + 2], acc[i][e + 3]);
    }
    if (ct == 0) {
      const bool any = it.r1 > it.r0;
      a.part_ml[item * 2] = SOFTMAX ? m : 0.f;
      a.part_ml[item * 2 + 1] = SOFTMAX ? l : (any ? 1.f : 0.f);
    }
  }
}

// Sparse plan: one CTA lists the items (pair * n_split + split) that hold rows -- routed chunk valid, weight
// non-zero, page inside the pool, split below the chunk's valid rows -- in item order, so that the read kernel's
// CTAs share only live work (a read where the selector masked most rows would otherwise leave most CTAs idle
// and a few with several items). Flags the device status as decode_item does for the pairs it skips.
constexpr int RC_THREADS = 1024;
__global__ void __launch_bounds__(RC_THREADS) read_compact_kernel(const ReadArgs a, int32_t* __restrict__ list,
                                                                  int* __restrict__ n_active) {
  __shared__ int wsum[RC_THREADS / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t pairs = a.n_rows * a.k;
  int total = 0;
  for (int64_t base = 0; base < pairs; base += blockDim.x) {
    const int64_t pr = base + threadIdx.x;
    int cnt = 0;
    if (pr < pairs) {
      const int32_t c = a.idx[pr];
      const float w = a.wk[pr];
      if (c >= 0 && c < a.n_chunks && w != 0.f) {
        const int64_t lc = (pr / a.k / a.rows_per_lib) * a.n_chunks + c;
        const int64_t page = a.page_of[lc];
        if (page < 0 || page >= a.n_pages) {
          flag_error(XENCB_DEV_BADPAGE);
        } else {
          int nv = a.n_valid[lc];
          if (nv > a.page_rows) { nv = a.page_rows; flag_error(XENCB_DEV_CLAMPED); }
          if (nv < 0) nv = 0;
          cnt = min(a.n_split, (nv + a.split_rows - 1) / a.split_rows);
        }
      }
    }
    // block-wide exclusive scan of cnt
    int x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int t = lane < nw ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      if (lane < nw) wsum[lane] = t;
    }
    __syncthreads();
    const int off = total + (wid > 0 ? wsum[wid - 1] : 0) + x - cnt;
    for (int sp = 0; sp < cnt; ++sp) list[off + sp] = (int32_t)(pr * a.n_split + sp);
    total += wsum[nw - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_active = total;
}

// r[row] = sum_j w_j * read_j; grid (n_rows, ceil(d_s / 512)), 128 threads x 4 columns.
// Entries of a row are its (chunk j, split s) items in that order, merged in batches of MERGE_ENTRIES. Each thread
// requests the partial vectors of its 4 columns for the batch's first MERGE_VEC entries at once, before the
// coefficients are known; meanwhile the batch's (m, l) pairs go to shared memory and one thread per chunk turns
// them into coefficients (log-sum-exp over the chunk's live splits, the routing weight, 1/l or 1/sqrt(n); 0 for an
// entry that takes no part, whose vector is never used). The sum runs in entry order, so it is deterministic.
constexpr int MERGE_THREADS = 128, MERGE_ENTRIES = 128, MERGE_VEC = 16;

__device__ __forceinline__ void fma4(float c, const float4& v, float4& r) {
  r.x = fmaf(c, v.x, r.x); r.y = fmaf(c, v.y, r.y); r.z = fmaf(c, v.z, r.z); r.w = fmaf(c, v.w, r.w);
}

template <bool SOFTMAX>
__global__ void __launch_bounds__(MERGE_THREADS) read_merge_kernel(const ReadArgs a, float* __restrict__ r_out) {
  __shared__ float ml[2 * MERGE_ENTRIES];
  __shared__ float coef[MERGE_ENTRIES];
  __shared__ int nan_flag;
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + tid) * 4;
  const bool colok = col < a.d_s;
  const int ns = a.n_split;
  const int jb_step = max(1, MERGE_ENTRIES / ns);  // chunks per batch
  const int64_t row_item0 = row * (int64_t)a.k * ns;
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid == 0) nan_flag = 0;
  for (int jb = 0; jb < a.k; jb += jb_step) {
    const int nj = min(jb_step, a.k - jb), ne = nj * ns;
    const int64_t e0 = row_item0 + (int64_t)jb * ns;
    const float* pa = a.part_acc + e0 * a.d_s + col;
    float4 v[MERGE_VEC];
    if (colok) {
#pragma unroll
      for (int u = 0; u < MERGE_VEC; ++u)
        if (u < ne) v[u] = __ldcg(reinterpret_cast<const float4*>(pa + (int64_t)u * a.d_s));
    }
    for (int e = tid; e < 2 * ne; e += blockDim.x) ml[e] = a.part_ml[e0 * 2 + e];
    __syncthreads();
    for (int jj = tid; jj < nj; jj += blockDim.x) {
      float* cf = coef + jj * ns;
      for (int s = 0; s < ns; ++s) cf[s] = 0.f;
      const int64_t pair = row * a.k + jb + jj;
      const int32_t c = a.idx[pair];
      const float w = a.wk[pair];
      if (c < 0 || c >= a.n_chunks || w == 0.f) continue;
      const int64_t lc = (row / a.rows_per_lib) * a.n_chunks + c;
      const int64_t page = a.page_of[lc];
      if (page < 0 || page >= a.n_pages) continue;  // skipped by the read (flagged there)
      int nv = a.n_valid[lc];
      nv = nv > a.page_rows ? a.page_rows : (nv < 0 ? 0 : nv);
      const int n_live = min(ns, (nv + a.split_rows - 1) / a.split_rows);  // splits holding rows
      const float* mj = ml + 2 * jj * ns;
      float M = -CUDART_INF_F, L = 0.f;
      if (SOFTMAX) {
        for (int s = 0; s < n_live; ++s)
          if (mj[2 * s + 1] > 0.f) M = fmaxf(M, mj[2 * s]);
        for (int s = 0; s < n_live; ++s) {
          const float ls = mj[2 * s + 1];
          if (ls > 0.f) L += ls * exp2f(mj[2 * s] - M);
        }
        if (!(L > 0.f)) {  // a routed chunk without a valid slot: the reference's softmax gives NaN
          atomicOr(&nan_flag, 1);
          continue;
        }
      } else {
        L = sqrtf((float)(nv > 1 ? nv : 1));
      }
      for (int s = 0; s < n_live; ++s)
        if (mj[2 * s + 1] > 0.f) cf[s] = SOFTMAX ? w * exp2f(mj[2 * s] - M) / L : w / L;
    }
    __syncthreads();
    if (colok) {
#pragma unroll
      for (int u = 0; u < MERGE_VEC; ++u) {
        if (u < ne) {
          const float cu = coef[u];
          if (cu != 0.f) fma4(cu, v[u], r);
        }
      }
      for (int eb = MERGE_VEC; eb < ne; eb += MERGE_VEC) {
#pragma unroll
        for (int u = 0; u < MERGE_VEC; ++u)
          if (eb + u < ne && coef[eb + u] != 0.f)
            v[u] = __ldcg(reinterpret_cast<const float4*>(pa + (int64_t)(eb + u) * a.d_s));
#pragma unroll
        for (int u = 0; u < MERGE_VEC; ++u) {
          if (eb + u < ne) {
            const float cu = coef[eb + u];
            if (cu != 0.f) fma4(cu, v[u], r);
          }
        }
      }
    }
    __syncthreads();
  }
  if (nan_flag) r = make_float4(CUDART_NAN_F, CUDART_NAN_F, CUDART_NAN_F, CUDART_NAN_F);
  if (colok) *reinterpret_cast<float4*>(r_out + row * (int64_t)a.d_s + col) = r;
}

}  // namespace xencb

// Many-query read over whole chunks (f16 / bf16 slots): up to 8 query rows of one Library share every slot row
// fetched from HBM. This is the dense read of a Library queried by several tokens at once
// (xenc/injector.py:239-265 with T > 1): every query row scores and accumulates every valid slot of every chunk
// it routes to, with per-(row, chunk) weights w[row, c] (0 = not routed; the softmax of the routing logits, or
// their unnormalised exponentials for a shard's partial).
//
// Work decomposition. A group is (Library, block of <= 8 of its query rows). Each chunk of a group is cut into
// `pieces` pieces of `piece_rows` rows; the units (group, chunk, piece) are numbered in that order and CTA b
// takes the contiguous range [b*U/grid, (b+1)*U/grid). A chunk whose units all fall in one CTA is complete
// there: at its end the CTA adds w[row, c] * acc / l for each query into the group's fold slot (a per-CTA
// accumulator in global memory, which stays in L2). A chunk cut by a range boundary leaves an open partial
// (m, l, acc) per query in the CTA's head or tail slot. read_multi_coef_kernel and read_multi_sum_kernel add, per
// group, the fold slots of the CTAs that cover it and the open partials (log-sum-exp merged per chunk, then
// weighted).
//
// CTA shape and the per-16-row arithmetic follow read_decode_mma_kernel: warp 0 lane 0 issues one 1-D bulk copy
// (TMA, no multicast) per slot row into padded shared-memory rows; consumer warp w owns the 16*TPW columns
// [16*TPW*w, 16*TPW*(w+1)) and runs
//   scores  S[16 rows x 8 queries]  += K[rows, 16 cols] (ldmatrix)     x Q[16 cols, 8 queries]
//   accum   A[16 cols x 8 queries]  += K^T[16 cols, rows] (ldmatrix.trans) x P[rows, 8 queries]
// with the partial scores summed across warps in a double-buffered shared array behind an mbarrier. Lane L
// finishes query L/4 on rows 2(L%4), 2(L%4)+1, 2(L%4)+8, 2(L%4)+9 of the group -- exactly the P values its
// B fragment of the second product needs, so P never moves between lanes.
// Every wait is bounded; a warp that gives up raises the abort flag and all others then leave.
#pragma once

#include "read_decode_mma.cuh"

namespace xencb {

constexpr int MQ = 8;          // query rows per group (the MMA's N)
constexpr int MQ_RED = 24;     // floats per query in the cross-warp score buffer (conflict-free float2 reads)
constexpr int MQ_OPEN = 2 * MQ;  // floats of (m, l) pairs at the start of an open slot

struct MultiArgs {
  const float* q;
  int64_t n_rows;
  int d_s;
  const char* slots;
  const char* vslots;  // untied values (same page layout), or null when V = K
  int64_t n_pages;
  int64_t page_stride_bytes;
  int page_rows;
  const int32_t* page_of;
  const int32_t* n_valid;
  int n_chunks;
  const int32_t* n_chunks_of;
  int64_t rows_per_lib;
  const float* w;  // [n_rows, n_chunks]
  float qscale;    // read_temp * log2(e) (softmax) or 1 (linear)
  int q_blocks;    // ceil(min(rows_per_lib, n_rows) / MQ) groups per Library
  int64_t n_groups;
  int pieces, piece_rows;
  int64_t units_per_group;  // n_chunks * pieces
  int64_t n_units;          // n_groups * units_per_group
  int s_max;                // fold slots per CTA
  int rps, n_stage, row_bytes, row_stride;
  float* fold;          // [grid][s_max][MQ][d_s]
  int64_t* fold_info;   // [grid][s_max]: group, or -1 when the slot holds nothing
  float* open;          // [grid][2][MQ_OPEN + MQ * d_s]: (m, l) per query, then acc per query
  int64_t* open_info;   // [grid][2]: group * n_chunks + chunk, or -1
  int* merge_counter;   // [n_groups * merge slabs], zeroed here for read_multi_sum_kernel
  int64_t n_merge_counters;
};

struct __align__(16) MultiMeta {
  int64_t g;
  int c, nv, nr, flags;
};
constexpr int MM_FIRST = 1, MM_LAST = 2, MM_DONE = 4, MM_HEAD = 8, MM_TAIL = 16, MM_PIECE0 = 32;
constexpr int MM_VAL = 64;  // a stage of value rows (untied V): the P of the preceding key stage times these rows

__host__ __device__ inline int64_t mq_unit_begin(int64_t b, int64_t n_units, int64_t grid) {
  return b * n_units / grid;
}
// the CTA whose range holds unit u
__host__ __device__ inline int64_t mq_cta_of(int64_t u, int64_t n_units, int64_t grid) {
  return ((u + 1) * grid - 1) / n_units;
}

__host__ __device__ inline size_t mq_smem_bytes(int n_stage, int stage_bytes, int ncw, int tpw, bool split) {
  return (size_t)n_stage * stage_bytes                     // stages
         + (size_t)ncw * (split ? 2 : 1) * tpw * 32 * 8      // q fragments (one uint2 per lane per tile)
         + 2 * (size_t)ncw * MQ * MQ_RED * 4                 // cross-warp partial scores
         + (size_t)n_stage * sizeof(MultiMeta)               // stage descriptors
         + (2 * (size_t)n_stage + 2) * 8                     // full / empty / two score barriers
         + 16;                                               // abort flag
}

template <typename T, bool SPLIT, bool SOFTMAX, int TPW>
__global__ void __launch_bounds__(TPW == 8 ? 32 * (RM_MAX_WARPS + 1) : 32 * 11, 1) read_multi_mma_kernel(const MultiArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = (blockDim.x >> 5) - 1;
  const int row_stride = a.row_stride;
  const int stage_bytes = ((a.rps * row_stride + 127) / 128) * 128;
  unsigned char* stages = smem;
  uint2* qfrag = reinterpret_cast<uint2*>(smem + (size_t)a.n_stage * stage_bytes);        // [ncw][1|2][TPW][32]
  float* red = reinterpret_cast<float*>(qfrag + (size_t)ncw * (SPLIT ? 2 : 1) * TPW * 32);  // [2][ncw][MQ*MQ_RED]
  MultiMeta* meta = reinterpret_cast<MultiMeta*>(red + 2 * ncw * MQ * MQ_RED);
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + a.n_stage);
  uint64_t* empty = full + a.n_stage;
  uint64_t* sbar = empty + a.n_stage;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sbar + 2);

  const int64_t u_begin = mq_unit_begin(blockIdx.x, a.n_units, gridDim.x);
  const int64_t u_end = mq_unit_begin(blockIdx.x + 1, a.n_units, gridDim.x);
  const int64_t g_first = u_begin / a.units_per_group;

  {
    uint4* z = reinterpret_cast<uint4*>(stages);
    const int n16 = a.n_stage * stage_bytes / 16;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) z[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.n_stage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], ncw);
    }
    mbar_init(&sbar[0], ncw);
    mbar_init(&sbar[1], ncw);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Under programmatic dependent launch the shared-memory set-up above overlaps the kernel before; global memory
  // is read and written only after the wait. The trigger lets the merge's first kernel be scheduled.
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < a.s_max; i += blockDim.x) a.fold_info[(int64_t)blockIdx.x * a.s_max + i] = -1;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n_merge_counters;
       i += (int64_t)gridDim.x * blockDim.x)
    a.merge_counter[i] = 0;
  if (threadIdx.x < 2) a.open_info[(int64_t)blockIdx.x * 2 + threadIdx.x] = -1;
  __syncthreads();

  // ------------------------------------------------------------------------------------------- producer
  if (warp == 0) {
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    uint32_t it_count = 0;
    bool ok = true;
    for (int64_t u = u_begin; u < u_end && ok;) {
      const int64_t g = u / a.units_per_group;
      const int64_t rem = u - g * a.units_per_group;
      const int c = (int)(rem / a.pieces);
      const int p0 = (int)(rem - (int64_t)c * a.pieces);
      const int64_t chunk_first = g * a.units_per_group + (int64_t)c * a.pieces;
      const int64_t chunk_end = chunk_first + a.pieces;
      const int64_t v_end = chunk_end < u_end ? chunk_end : u_end;
      const int p1 = (int)(v_end - chunk_first);
      u = v_end;
      const bool head = chunk_first < u_begin;
      const bool tail = !head && chunk_end > u_end;
      const int64_t lib = g / a.q_blocks;
      const int64_t row0 = lib * a.rows_per_lib + (g - lib * a.q_blocks) * MQ;
      int64_t row_lim = lib * a.rows_per_lib + a.rows_per_lib;
      if (row_lim > a.n_rows) row_lim = a.n_rows;
      const int nq = (int)(row_lim - row0 < MQ ? row_lim - row0 : MQ);
      const int nc = a.n_chunks_of ? a.n_chunks_of[lib] : a.n_chunks;
      if (nq <= 0 || c >= nc) continue;
      bool any = false;
      for (int j = 0; j < nq; ++j) any |= a.w[(row0 + j) * a.n_chunks + c] != 0.f;
      if (!any) continue;
      const int64_t lc = lib * a.n_chunks + c;
      const int64_t page = a.page_of[lc];
      if (page < 0 || page >= a.n_pages) {  // never read outside the pool
        flag_error(XENCB_DEV_BADPAGE);
        continue;
      }
      int nv = a.n_valid[lc];
      if (nv > a.page_rows) { nv = a.page_rows; flag_error(XENCB_DEV_CLAMPED); }
      const int r0 = p0 * a.piece_rows;
      const int r1 = min(nv, p1 * a.piece_rows);
      if (r1 <= r0) continue;
      const char* base = a.slots + page * a.page_stride_bytes;
      for (int rs = r0; rs < r1 && ok; rs += a.rps) {
        const int nr = min(a.rps, r1 - rs);
        const int visit = (head ? MM_HEAD : 0) | (tail ? MM_TAIL : 0) | (p0 == 0 ? MM_PIECE0 : 0);
        const bool last = rs + nr >= r1;
        // key rows, then (untied values) the same rows of the value pool as the next stage
        for (int part = 0; part < (a.vslots ? 2 : 1); ++part) {
          const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
          if (use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) { ok = false; break; }
          meta[slot].g = g;
          meta[slot].c = c;
          meta[slot].nv = nv;
          meta[slot].nr = nr;
          meta[slot].flags = visit | (part == 0 ? ((rs == r0 ? MM_FIRST : 0) | (last && !a.vslots ? MM_LAST : 0))
                                                : (MM_VAL | (last ? MM_LAST : 0)));
          mbar_arrive_expect_tx(&full[slot], (uint32_t)nr * a.row_bytes);
          unsigned char* dst = stages + (size_t)slot * stage_bytes;
          const char* src = (part == 0 ? base : a.vslots + (base - a.slots)) + (int64_t)rs * a.row_bytes;
          for (int r = 0; r < nr; ++r)
            bulk_g2s(dst + (size_t)r * row_stride, src + (int64_t)r * a.row_bytes, (uint32_t)a.row_bytes,
                     &full[slot], pol);
          ++it_count;
        }
      }
    }
    if (ok) {
      const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
      if (use == 0 || mbar_wait_bounded(&empty[slot], (use - 1) & 1)) {
        meta[slot].g = -1;
        meta[slot].nr = 0;
        meta[slot].flags = MM_DONE;
        mbar_arrive(&full[slot]);
        ++it_count;
      }
    }
    const uint32_t n_slots = it_count < (uint32_t)a.n_stage ? it_count : (uint32_t)a.n_stage;
    for (uint32_t i = 0; i < n_slots; ++i) {
      const uint32_t last = it_count - 1 - i;
      mbar_wait_bounded(&full[last % a.n_stage], (last / a.n_stage) & 1);
    }
    return;
  }

  // ------------------------------------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int d0 = cw * (16 * TPW);
  const int nt = min(TPW, (a.d_s - d0) / 16);
  uint2* qf = qfrag + (size_t)cw * (SPLIT ? 2 : 1) * TPW * 32;
  const uint32_t stages_u32 = smem_u32(stages);
  const int mtx = lane >> 3, r8 = lane & 7;
  const uint32_t off_s = (uint32_t)((r8 + (mtx & 1) * 8) * row_stride + (mtx >> 1) * 16 + d0 * 2);
  const uint32_t off_a = (uint32_t)((r8 + (mtx >> 1) * 8) * row_stride + (mtx & 1) * 16 + d0 * 2);
  const int qj = lane >> 2;        // query this lane finishes
  const int i0 = (lane & 3) * 2;   // its rows i0, i0+1, i0+8, i0+9 of a 16-row group
  const int qa = (lane & 3) * 2;   // accumulator columns (queries) qa, qa+1 of this lane
  const int rl = lane >> 2;        // accumulator fragment rows rl, rl+8 (columns of d)

  float acc[TPW][4];
  float m = -CUDART_INF_F, l = 0.f;
  int64_t cur_g = -1, row0 = 0;
  int nq = 0;
  bool fold_any = false;
  uint32_t it_count = 0, grp = 0;
  uint32_t vb0 = 0u, vb1 = 0u, vc0 = 0u, vc1 = 0u;  // P fragments of the last key group (untied values)
  // end of a chunk visit: fold a complete chunk into the group's slot, or write an open slot
  auto finish_visit = [&](const MultiMeta& md) {
      const bool open = (md.flags & (MM_HEAD | MM_TAIL)) != 0;
      const float inv_sqrt_n = SOFTMAX ? 1.f : 1.f / sqrtf((float)md.nv);
      if (!open) {
        // complete chunk: fold w * acc / l into the group's slot (each lane owns its elements, so the
        // read-modify-write needs no synchronisation)
        float f = 0.f;
        if (qj < nq) {
          const float wq = a.w[(row0 + qj) * a.n_chunks + md.c];
          f = SOFTMAX ? (l > 0.f ? wq / l : 0.f) : wq * inv_sqrt_n;
        }
        const float f_a = __shfl_sync(0xffffffffu, f, qa * 4);
        const float f_b = __shfl_sync(0xffffffffu, f, qa * 4 + 4);
        const int64_t seg = md.g - g_first;
        float* fs = a.fold + ((int64_t)blockIdx.x * a.s_max + seg) * MQ * a.d_s;
        float* fa = fs + (int64_t)qa * a.d_s;
        float* fb = fa + a.d_s;
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          if (t < nt) {
            const int d = d0 + t * 16 + rl;
            float x0 = acc[t][0] * f_a, x1 = acc[t][1] * f_b, x2 = acc[t][2] * f_a, x3 = acc[t][3] * f_b;
            if (fold_any) {
              x0 += fa[d]; x1 += fb[d]; x2 += fa[d + 8]; x3 += fb[d + 8];
            }
            fa[d] = x0; fb[d] = x1; fa[d + 8] = x2; fb[d + 8] = x3;
          }
        }
        if (!fold_any && cw == 0 && lane == 0) a.fold_info[(int64_t)blockIdx.x * a.s_max + seg] = md.g;
        fold_any = true;
      } else {
        const int oslot = (md.flags & MM_HEAD) ? 0 : 1;
        float* os = a.open + ((int64_t)blockIdx.x * 2 + oslot) * (MQ_OPEN + (int64_t)MQ * a.d_s);
        float* oa = os + MQ_OPEN + (int64_t)qa * a.d_s;
        float* ob = oa + a.d_s;
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          if (t < nt) {
            const int d = d0 + t * 16 + rl;
            oa[d] = acc[t][0] * inv_sqrt_n;
            ob[d] = acc[t][1] * inv_sqrt_n;
            oa[d + 8] = acc[t][2] * inv_sqrt_n;
            ob[d + 8] = acc[t][3] * inv_sqrt_n;
          }
        }
        if (cw == 0 && (lane & 3) == 0) {
          os[qj * 2] = SOFTMAX ? m : 0.f;
          os[qj * 2 + 1] = SOFTMAX ? l : ((md.flags & MM_PIECE0) ? 1.f : 0.f);
        }
        if (cw == 0 && lane == 0) a.open_info[(int64_t)blockIdx.x * 2 + oslot] = md.g * a.n_chunks + md.c;
      }
  };


  while (true) {
    const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
    ++it_count;
    if (!mbar_wait_bounded(&full[slot], use & 1) || *abort_flag) { *abort_flag = 1; break; }
    const MultiMeta md = meta[slot];
    if (md.flags & MM_DONE) break;

    if (md.flags & MM_VAL) {
      const uint32_t vbase = stages_u32 + slot * (uint32_t)stage_bytes;
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (t < nt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vbase + off_a + t * 32, a0, a1, a2, a3);
          mma16816<T>(acc[t], a0, a1, a2, a3, vb0, vb1);
          if (SPLIT) mma16816<T>(acc[t], a0, a1, a2, a3, vc0, vc1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (md.flags & MM_LAST) finish_visit(md);
      continue;
    }

    if (md.flags & MM_FIRST) {
      if (md.g != cur_g) {
        cur_g = md.g;
        fold_any = false;
        const int64_t lib = cur_g / a.q_blocks;
        row0 = lib * a.rows_per_lib + (cur_g - lib * a.q_blocks) * MQ;
        int64_t row_lim = lib * a.rows_per_lib + a.rows_per_lib;
        if (row_lim > a.n_rows) row_lim = a.n_rows;
        nq = (int)(row_lim - row0 < MQ ? row_lim - row0 : MQ);
        // B fragments of the score product: lane holds Q[cols i0, i0+1 | i0+8, i0+9 of tile t][query qj]
        const bool has = qj < nq;
        const float* qr = a.q + (row0 + (has ? qj : 0)) * a.d_s;
        for (int t = 0; t < nt; ++t) {
          const int k = d0 + t * 16 + i0;
          const float x0 = has ? __ldg(qr + k) * a.qscale : 0.f, x1 = has ? __ldg(qr + k + 1) * a.qscale : 0.f;
          const float x2 = has ? __ldg(qr + k + 8) * a.qscale : 0.f, x3 = has ? __ldg(qr + k + 9) * a.qscale : 0.f;
          float h0, h1, h2, h3, l0, l1, l2, l3;
          uint2 hi, lo;
          hi.x = pack2<T>(x0, x1, h0, h1);
          hi.y = pack2<T>(x2, x3, h2, h3);
          qf[t * 32 + lane] = hi;
          if (SPLIT) {
            lo.x = pack2<T>(x0 - h0, x1 - h1, l0, l1);
            lo.y = pack2<T>(x2 - h2, x3 - h3, l2, l3);
            qf[(TPW + t) * 32 + lane] = lo;
          }
        }
        __syncwarp();
      }
#pragma unroll
      for (int t = 0; t < TPW; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
      m = -CUDART_INF_F;
      l = 0.f;
    }
    const uint32_t sbase = stages_u32 + slot * (uint32_t)stage_bytes;
    bool aborted = false;

    for (int g0 = 0; g0 < md.nr; g0 += 16) {
      const int gv = min(16, md.nr - g0);
      const uint32_t gbase = sbase + (uint32_t)(g0 * row_stride);
      float sa[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) sa[c][0] = sa[c][1] = sa[c][2] = sa[c][3] = 0.f;
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (t < nt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(gbase + off_s + t * 32, a0, a1, a2, a3);
          const uint2 b = qf[t * 32 + lane];
          mma16816<T>(sa[t & 3], a0, a1, a2, a3, b.x, b.y);
          if (SPLIT) {
            const uint2 bl = qf[(TPW + t) * 32 + lane];
            mma16816<T>(sa[(t + 2) & 3], a0, a1, a2, a3, bl.x, bl.y);
          }
        }
      }
      // partial scores S[row rl | rl+8][query qa | qa+1] of this warp's columns
      const float s00 = (sa[0][0] + sa[1][0]) + (sa[2][0] + sa[3][0]);
      const float s01 = (sa[0][1] + sa[1][1]) + (sa[2][1] + sa[3][1]);
      const float s10 = (sa[0][2] + sa[1][2]) + (sa[2][2] + sa[3][2]);
      const float s11 = (sa[0][3] + sa[1][3]) + (sa[2][3] + sa[3][3]);
      const int b = grp & 1;
      float* rb = red + (size_t)b * ncw * MQ * MQ_RED;
      {
        float* mine = rb + cw * MQ * MQ_RED;
        mine[qa * MQ_RED + rl] = s00;
        mine[(qa + 1) * MQ_RED + rl] = s01;
        mine[qa * MQ_RED + rl + 8] = s10;
        mine[(qa + 1) * MQ_RED + rl + 8] = s11;
      }
      __syncwarp();
      if (ncw > 1) {
        if (lane == 0) mbar_arrive(&sbar[b]);
        if (!mbar_wait_bounded(&sbar[b], (grp >> 1) & 1) || *abort_flag) {
          *abort_flag = 1;
          aborted = true;
          break;
        }
      }
      ++grp;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      for (int w = 0; w < ncw; ++w) {
        const float* src = rb + w * MQ * MQ_RED + qj * MQ_RED + i0;
        const float2 lo2 = *reinterpret_cast<const float2*>(src);
        const float2 hi2 = *reinterpret_cast<const float2*>(src + 8);
        v[0] += lo2.x; v[1] += lo2.y; v[2] += hi2.x; v[3] += hi2.y;
      }
      if (ncw == 1) __syncwarp();  // the single warp re-writes this buffer two groups later
      const bool ok0 = i0 < gv, ok1 = i0 + 1 < gv, ok8 = i0 + 8 < gv, ok9 = i0 + 9 < gv;
      float p[4];
      if (SOFTMAX) {
        float mx = fmaxf(fmaxf(ok0 ? v[0] : -CUDART_INF_F, ok1 ? v[1] : -CUDART_INF_F),
                         fmaxf(ok8 ? v[2] : -CUDART_INF_F, ok9 ? v[3] : -CUDART_INF_F));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m, mx);
        const bool grew = m_new != m;
        const float sc = grew ? exp2f(m - m_new) : 1.f;
        if (__any_sync(0xffffffffu, grew)) {
          const float sc_a = __shfl_sync(0xffffffffu, sc, qa * 4);
          const float sc_b = __shfl_sync(0xffffffffu, sc, qa * 4 + 4);
#pragma unroll
          for (int t = 0; t < TPW; ++t) {
            acc[t][0] *= sc_a;
            acc[t][1] *= sc_b;
            acc[t][2] *= sc_a;
            acc[t][3] *= sc_b;
          }
        }
        l *= sc;
        m = m_new;
        p[0] = ok0 ? exp2f(v[0] - m) : 0.f;
        p[1] = ok1 ? exp2f(v[1] - m) : 0.f;
        p[2] = ok8 ? exp2f(v[2] - m) : 0.f;
        p[3] = ok9 ? exp2f(v[3] - m) : 0.f;
      } else {
        p[0] = ok0 ? v[0] : 0.f;
        p[1] = ok1 ? v[1] : 0.f;
        p[2] = ok8 ? v[2] : 0.f;
        p[3] = ok9 ? v[3] : 0.f;
      }
      // round p to the slot type (+ residual for bf16); l sums the values the MMA uses
      float ph[4], pl[4];
      uint32_t pb0, pb1, pc0 = 0u, pc1 = 0u;
      pb0 = pack2<T>(p[0], p[1], ph[0], ph[1]);
      pb1 = pack2<T>(p[2], p[3], ph[2], ph[3]);
      if (SPLIT) {
        pc0 = pack2<T>(p[0] - ph[0], p[1] - ph[1], pl[0], pl[1]);
        pc1 = pack2<T>(p[2] - ph[2], p[3] - ph[3], pl[2], pl[3]);
      }
      if (SOFTMAX) {
        float ps = (ph[0] + ph[1]) + (ph[2] + ph[3]);
        if (SPLIT) ps += (pl[0] + pl[1]) + (pl[2] + pl[3]);
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        l += ps;
      }
      if (a.vslots) {  // untied: the value stage that follows does the accumulation (one group per stage)
        vb0 = pb0; vb1 = pb1; vc0 = pc0; vc1 = pc1;
        continue;
      }
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (t < nt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(gbase + off_a + t * 32, a0, a1, a2, a3);
          mma16816<T>(acc[t], a0, a1, a2, a3, pb0, pb1);
          if (SPLIT) mma16816<T>(acc[t], a0, a1, a2, a3, pc0, pc1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (aborted) break;
    if (md.flags & MM_LAST) finish_visit(md);
  }
}



// r[row] = sum of the fold slots of the CTAs covering the row's group + the open partials, merged per chunk
// (log2-domain log-sum-exp) and weighted by w[row, c]. Because the merge of a chunk's pieces is a weighted sum
// with per-(piece, query) coefficients w_c 2^(m_p - M) / L that do not depend on the column, every output is
//     r[q][d] = sum_src coef[src][q] * data[src][q][d]        (coef = 1 for fold slots)
// Two kernels:
//   read_multi_coef_kernel (one CTA per group): warp 0 compacts the group's fold slots and open slots (unit
//     order) and cuts the open slots into runs of one chunk; the threads compute the runs' coefficients; the
//     result is the group's source list (float offset + 8 coefficients per source);
//   read_multi_sum_kernel (grid groups x 128-column slabs x MM_SQ): each CTA sums its share of the sources with
//     float4 loads (warps split the sources, lane = 4 columns, 8 float4 accumulators) into a block partial; the
//     last CTA of a (group, slab) adds the MM_SQ partials in a fixed order and writes r. The per-slab counters
//     are zeroed by read_multi_mma_kernel (stream order) and re-armed by the last CTA.
constexpr int MM_MERGE_THREADS = 256;
constexpr int MM_MERGE_WARPS = MM_MERGE_THREADS / 32;
constexpr int MM_SQ = 8;                  // source splits per (group, slab)
constexpr int MM_MERGE_MAX_CTAS = 160;    // read grids up to this many CTAs (static shared memory < 48 KB)
constexpr int MM_MERGE_MAX_SLOTS = 2 * MM_MERGE_MAX_CTAS;
constexpr int MM_SRC_PER_CTA = 3;         // sources per read CTA at most: one fold slot + two open slots

struct MultiMergeArgs {
  float* part;        // [n_groups][n_slabs][MM_SQ][MQ][128]
  int* counter;       // [n_groups][n_slabs]
  int64_t* src_off;   // [n_groups][MM_SRC_PER_CTA * grid]: float offset from a.fold (>= 0) or ~offset from a.open
  float* src_coef;    // [n_groups][MM_SRC_PER_CTA * grid][MQ]
  int* src_count;     // [n_groups]
  int n_slabs;
};

template <bool SOFTMAX>
__global__ void __launch_bounds__(MM_MERGE_THREADS) read_multi_coef_kernel(const MultiArgs a, int grid,
                                                                           MultiMergeArgs mm) {
  __shared__ int slot_of[MM_MERGE_MAX_SLOTS];
  __shared__ int run_start[MM_MERGE_MAX_SLOTS + 1];
  __shared__ int fold_of[MM_MERGE_MAX_CTAS];
  __shared__ int n_open, n_runs, n_fold;
  pdl_wait();
  pdl_trigger();
  const int64_t g = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t lib = g / a.q_blocks;
  const int64_t row0 = lib * a.rows_per_lib + (g - lib * a.q_blocks) * MQ;
  int64_t row_lim = lib * a.rows_per_lib + a.rows_per_lib;
  if (row_lim > a.n_rows) row_lim = a.n_rows;
  const int nq = (int)(row_lim - row0 < MQ ? row_lim - row0 : MQ);
  const int cap = MM_SRC_PER_CTA * grid;
  int64_t* so = mm.src_off + g * cap;
  float* sc = mm.src_coef + g * cap * MQ;
  if (nq <= 0) {
    if (threadIdx.x == 0) mm.src_count[g] = 0;
    return;
  }
  const int64_t b0 = mq_cta_of(g * a.units_per_group, a.n_units, grid);
  const int64_t b1 = mq_cta_of((g + 1) * a.units_per_group - 1, a.n_units, grid);
  const int n_cta = (int)(b1 - b0 + 1);
  // every slot's info in one parallel pass (independent loads), then warp 0 scans shared memory
  __shared__ int64_t oinfo_s[MM_MERGE_MAX_SLOTS];
  __shared__ unsigned char fok_s[MM_MERGE_MAX_CTAS];
  for (int i = threadIdx.x; i < n_cta; i += blockDim.x) {
    const int64_t b = b0 + i;
    const int64_t seg = g - mq_unit_begin(b, a.n_units, grid) / a.units_per_group;
    fok_s[i] = (seg >= 0 && seg < a.s_max && a.fold_info[b * a.s_max + seg] == g) ? 1 : 0;
  }
  for (int i = threadIdx.x; i < 2 * n_cta; i += blockDim.x) oinfo_s[i] = a.open_info[b0 * 2 + i];
  __syncthreads();
  if (warp == 0) {
    int cnt = 0;
    for (int base = 0; base < n_cta; base += 32) {
      const int i = base + lane;
      const bool mine = i < n_cta && fok_s[i];
      const unsigned m = __ballot_sync(0xffffffffu, mine);
      if (mine) fold_of[cnt + __popc(m & ((1u << lane) - 1u))] = i;
      cnt += __popc(m);
    }
    int oc = 0;
    for (int base = 0; base < 2 * n_cta; base += 32) {
      const int i = base + lane;
      const bool mine = i < 2 * n_cta && oinfo_s[i] >= 0 && oinfo_s[i] / a.n_chunks == g;
      const unsigned m = __ballot_sync(0xffffffffu, mine);
      if (mine) slot_of[oc + __popc(m & ((1u << lane) - 1u))] = i;  // index into oinfo_s (slot b0 * 2 + i)
      oc += __popc(m);
    }
    __syncwarp();
    int nr = 0;
    for (int base = 0; base < oc; base += 32) {
      const int i = base + lane;
      bool start = false;
      if (i < oc) start = i == 0 || oinfo_s[slot_of[i]] != oinfo_s[slot_of[i - 1]];
      const unsigned m = __ballot_sync(0xffffffffu, start);
      if (start) run_start[nr + __popc(m & ((1u << lane) - 1u))] = i;
      nr += __popc(m);
    }
    if (lane == 0) {
      run_start[nr] = oc;
      n_fold = cnt;
      n_open = oc;
      n_runs = nr;
      mm.src_count[g] = cnt + oc;
    }
  }
  __syncthreads();
  // fold sources: coefficient 1
  for (int i = threadIdx.x; i < n_fold; i += blockDim.x) {
    const int64_t b = b0 + fold_of[i];
    const int64_t seg = g - mq_unit_begin(b, a.n_units, grid) / a.units_per_group;
    so[i] = (b * a.s_max + seg) * MQ * a.d_s;
#pragma unroll
    for (int j = 0; j < MQ; ++j) sc[(int64_t)i * MQ + j] = 1.f;
  }
  // open sources: the slots' (m, l) pairs and the runs' routing weights in parallel passes, then one
  // (run, query) per thread from shared memory
  __shared__ __align__(16) float ml_s[MM_MERGE_MAX_SLOTS][MQ_OPEN];
  __shared__ float w_s[MM_MERGE_MAX_SLOTS][MQ];
  {
    // four 16-byte loads in flight per thread before any store (the (m, l) block of a slot is 64 bytes)
    constexpr int PER = 4;
    const int n4 = n_open * (MQ_OPEN / 4);
    for (int base = threadIdx.x; base < n4; base += blockDim.x * PER) {
      float4 v[PER];
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int t = base + u * blockDim.x;
        if (t < n4) {
          const int e = t / (MQ_OPEN / 4), k4 = t - e * (MQ_OPEN / 4);
          v[u] = __ldcg(reinterpret_cast<const float4*>(a.open + (b0 * 2 + slot_of[e]) * (MQ_OPEN + (int64_t)MQ * a.d_s)) + k4);
        }
      }
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int t = base + u * blockDim.x;
        if (t < n4) {
          const int e = t / (MQ_OPEN / 4), k4 = t - e * (MQ_OPEN / 4);
          reinterpret_cast<float4*>(ml_s[e])[k4] = v[u];
        }
      }
    }
  }
  for (int t = threadIdx.x; t < n_runs * MQ; t += blockDim.x) {
    const int rr = t / MQ, j = t - rr * MQ;
    const int c = (int)(oinfo_s[slot_of[run_start[rr]]] - g * a.n_chunks);
    w_s[rr][j] = j < nq ? a.w[(row0 + j) * a.n_chunks + c] : 0.f;
  }
  __syncthreads();
  for (int t = threadIdx.x; t < n_runs * MQ; t += blockDim.x) {
    const int rr = t / MQ, j = t - rr * MQ;
    const int e0 = run_start[rr], e1 = run_start[rr + 1];
    float Mx = -CUDART_INF_F, L = 0.f;
    for (int e = e0; e < e1; ++e) {
      const float mp = ml_s[e][j * 2], lp = ml_s[e][j * 2 + 1];
      if (SOFTMAX) {
        if (lp > 0.f) {
          const float mn = fmaxf(Mx, mp);
          L = L * exp2f(Mx - mn) + lp * exp2f(mp - mn);
          Mx = mn;
        }
      } else {
        L += lp;
      }
    }
    const float wl = (j < nq && L > 0.f) ? w_s[rr][j] / L : 0.f;
    for (int e = e0; e < e1; ++e) {
      float cf = 0.f;
      if (wl != 0.f) cf = SOFTMAX ? (ml_s[e][j * 2 + 1] > 0.f ? wl * exp2f(ml_s[e][j * 2] - Mx) : 0.f) : wl;
      sc[(int64_t)(n_fold + e) * MQ + j] = cf;
      if (j == 0)
        so[n_fold + e] = ~((b0 * 2 + slot_of[e]) * (MQ_OPEN + (int64_t)MQ * a.d_s) + MQ_OPEN);
    }
  }
}

__global__ void __launch_bounds__(MM_MERGE_THREADS, 2) read_multi_sum_kernel(const MultiArgs a, int grid,
                                                                             MultiMergeArgs mm,
                                                                             float* __restrict__ r_out) {
  __shared__ float4 red[MM_MERGE_WARPS][MQ][32];
  __shared__ int is_last;
  pdl_wait();
  pdl_trigger();
  const int64_t g = blockIdx.x;
  const int slab = blockIdx.y, sq = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = slab * 128 + lane * 4;
  const bool dok = d < a.d_s;  // d_s % 16 == 0: a float4 is either fully in or fully out
  const int64_t lib = g / a.q_blocks;
  const int64_t row0 = lib * a.rows_per_lib + (g - lib * a.q_blocks) * MQ;
  int64_t row_lim = lib * a.rows_per_lib + a.rows_per_lib;
  if (row_lim > a.n_rows) row_lim = a.n_rows;
  const int nq = (int)(row_lim - row0 < MQ ? row_lim - row0 : MQ);
  if (nq <= 0) return;  // uniform per (group): no counter of this group is ever armed
  const int cap = MM_SRC_PER_CTA * grid;
  const int64_t* so = mm.src_off + g * cap;
  const float* sc = mm.src_coef + g * cap * MQ;
  const int ns = mm.src_count[g];
  const int s_beg = (int)((int64_t)ns * sq / MM_SQ), s_end = (int)((int64_t)ns * (sq + 1) / MM_SQ);
  float4 acc[MQ];
#pragma unroll
  for (int j = 0; j < MQ; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (dok) {
    for (int si = s_beg + warp; si < s_end; si += MM_MERGE_WARPS) {
      const int64_t off = so[si];
      const float* base = off >= 0 ? a.fold + off : a.open + ~off;
      const float* cf = sc + (int64_t)si * MQ;
      float4 v[MQ];
#pragma unroll
      for (int j = 0; j < MQ; ++j)
        v[j] = j < nq ? *reinterpret_cast<const float4*>(base + (int64_t)j * a.d_s + d) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < MQ; ++j) {
        const float k = cf[j];
        acc[j].x = fmaf(k, v[j].x, acc[j].x);
        acc[j].y = fmaf(k, v[j].y, acc[j].y);
        acc[j].z = fmaf(k, v[j].z, acc[j].z);
        acc[j].w = fmaf(k, v[j].w, acc[j].w);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < MQ; ++j) red[warp][j][lane] = acc[j];
  __syncthreads();
  const int64_t pbase = ((g * mm.n_slabs + slab) * MM_SQ) * (int64_t)(MQ * 128);
  {
    const int j = threadIdx.x >> 5;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < MM_MERGE_WARPS; ++w) {
      const float4 x = red[w][j][lane];
      v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
    }
    *reinterpret_cast<float4*>(mm.part + pbase + (int64_t)sq * (MQ * 128) + j * 128 + lane * 4) = v;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(&mm.counter[g * mm.n_slabs + slab], 1) == MM_SQ - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  {
    const int j = threadIdx.x >> 5;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int z = 0; z < MM_SQ; ++z) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(mm.part + pbase + (int64_t)z * (MQ * 128) + j * 128 + lane * 4));
      v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
    }
    if (j < nq && dok) *reinterpret_cast<float4*>(r_out + (row0 + j) * a.d_s + d) = v;
  }
  if (threadIdx.x == 0) mm.counter[g * mm.n_slabs + slab] = 0;  // re-armed for the next call
}
static_assert(MM_MERGE_THREADS == 32 * MQ, "the block partial maps one query per warp");

// Shard merge: parts [G][n_rows * 4 + n_rows * d_s], per shard the rows' headers (max, sum, 0, 0) of the routing
// logits followed by the rows' accumulators A_g = sum_c e^(l_c - max) r_c. With M = max_g max_g:
//   r = sum_g e^(max_g - M) A_g / sum_g e^(max_g - M) sum_g         (natural-log domain, like the routing softmax)
// A shard whose sum is 0 (no chunk for that row) contributes nothing.
__global__ void __launch_bounds__(256) shard_merge_kernel(const float* __restrict__ parts, int G, int64_t n_rows,
                                                          int d_s, float* __restrict__ r_out) {
  const int64_t row = blockIdx.x;
  const int64_t per = n_rows * 4 + n_rows * (int64_t)d_s;
  float Mx = -CUDART_INF_F;
  for (int g = 0; g < G; ++g) Mx = fmaxf(Mx, parts[g * per + row * 4]);
  float den = 0.f;
  for (int g = 0; g < G; ++g) {
    const float* h = parts + g * per + row * 4;
    if (h[1] > 0.f) den += expf(h[0] - Mx) * h[1];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int d = blockIdx.y * blockDim.x + threadIdx.x; d < d_s; d += gridDim.y * blockDim.x) {
    float num = 0.f;
    for (int g = 0; g < G; ++g) {
      const float* h = parts + g * per + row * 4;
      if (h[1] > 0.f) num += expf(h[0] - Mx) * parts[g * per + n_rows * 4 + row * d_s + d];
    }
    r_out[row * d_s + d] = num * inv;
  }
}

}  // namespace xencb

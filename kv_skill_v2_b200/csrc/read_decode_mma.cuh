// Tensor-core decode read (f16 / bf16 slots): the same work items and partial format as read_decode_kernel,
// with the per-row arithmetic on mma.sync.m16n8k16.
//
// Producer (warp 0): decodes each work item once (page, valid rows), then per stage of `rps` rows lane 0
// writes a small descriptor (item, rows, first/last flags) into a shared ring and the warp's lanes bulk-copy
// (TMA, no multicast) the rows, one copy per row issued by lane row % 32, into the stage, rows padded by 16 bytes so the eight row addresses of an
// ldmatrix fall in distinct banks. A final descriptor marks the end of the CTA's work.
// Consumers (warps 1..ncw): warp w owns the (16*TPW)-column slice [16*TPW*w, 16*TPW*(w+1)) of d_s. Per
// 16-row group:
//   scores  S[16 x 8]  += K[rows, 16 cols] (ldmatrix)        x q[16 cols, query in column 0]   (TPW MMAs, 4 chains)
//   cross-warp sum of the 16 partial scores through a double-buffered shared array guarded by an mbarrier,
//   online softmax in fp32 (exp2 domain)
//   accum   A[16d x 8] += K^T[16d, rows] (ldmatrix.trans)    x p[rows, column 0]              (TPW MMAs)
// The same shared-memory tile feeds both products (K = V). q and p are rounded to the slot type (bf16 adds a
// residual term to both, so its products carry about 16 mantissa bits); accumulation is fp32.
// Rows past a group's valid count get p = 0; the ring is zeroed at start so those rows hold finite values.
// Every wait is an mbarrier wait with a time limit; a warp that gives up raises the abort flag and leaves,
// and every other wait then ends by itself, so no thread can be left waiting forever.
#pragma once

#include "read_decode.cuh"

namespace xencb {

constexpr int RM_TILES = 16;      // upper bound of the 16-column k-tiles per consumer warp (TPW <= RM_TILES)
constexpr int RM_MAX_WARPS = 16;  // consumer warps per CTA
constexpr int RM_RED_STRIDE = 20;  // floats per row of the cross-warp score buffer (>= RM_MAX_WARPS, 16-byte rows)
constexpr int RM_SBUF = 4;         // score buffers: a group's scores are posted one group before they are used

struct __align__(16) StageMeta {
  long long item;
  int nr;     // rows in this stage
  int flags;  // RM_FIRST | RM_LAST | RM_DONE
  long long row;       // the item's query row
  long long next_row;  // the query row of the CTA's next item when the producer has it decoded, else -1
};
constexpr int RM_FIRST = 1, RM_LAST = 2, RM_DONE = 4, RM_VAL = 8;  // RM_VAL: a stage of value rows (untied V)

// One posted 16-row group, as the consumers describe it to the softmax warp.
struct __align__(16) GroupRec {
  long long item;
  int flags;  // RM_FIRST on an item's first group, RM_LAST on its last, RM_DONE after the CTA's last group
  int gv;     // valid rows of the group
};

// Shared-memory bytes of the tensor-core read for a plan (the host and the kernel use the same layout).
// Item of work unit w: the listed item (sparse plan from read_compact_kernel), the in-kernel plan (the pair p with
// plan[p] <= w < plan[p + 1], plan = exclusive prefix sums of the pairs' live pieces, and its piece w - plan[p]),
// or w itself (dense plan).
__device__ __forceinline__ int64_t work_item(const ReadArgs& a, const int* plan, int64_t w) {
  if (a.item_list) return a.item_list[w];
  if (a.plan_pairs > 0) {
    int lo = 0, hi = a.plan_pairs;  // plan[lo] <= w < plan[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (plan[mid] <= w) lo = mid;
      else hi = mid;
    }
    return (int64_t)lo * a.n_split + (w - plan[lo]);
  }
  return w;
}

__host__ __device__ inline size_t rm_smem_bytes(int n_stage, int stage_bytes, int ncw, int tpw) {
  return (size_t)n_stage * stage_bytes           // stages
         + (size_t)ncw * 2 * tpw * 4 * 2 * 4       // q fragments
         + (size_t)ncw * 32 * (tpw / 8) * 16        // the next item's q, copied ahead [ncw][tpw / 8][32 lanes]
         + RM_SBUF * (size_t)16 * RM_RED_STRIDE * 4  // cross-warp partial scores [RM_SBUF][16 rows][stride]
         + (size_t)n_stage * sizeof(StageMeta)      // stage descriptors
         + RM_SBUF * sizeof(GroupRec)               // group records (consumers -> softmax warp)
         + RM_SBUF * (size_t)(4 * 4 + 4) * 4         // P fragments [4 lanes][4 words] + rescale factor
         + (2 * (size_t)n_stage + 2 * RM_SBUF) * 8  // full / empty / score / P barriers
         + 16;                                      // abort flag
}

template <typename T, bool SPLIT, bool SOFTMAX, int TPW>
__global__ void __launch_bounds__(TPW == 8 ? 32 * (RM_MAX_WARPS + 2) : 32 * 12, 1) read_decode_mma_kernel(const ReadArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = (blockDim.x >> 5) - 2;  // warp 0 producer, warps 1..ncw consumers, warp ncw + 1 softmax
  const int row_stride = a.row_stride;
  const int stage_bytes = ((a.rps * row_stride + 127) / 128) * 128;
  unsigned char* stages = smem;
  uint32_t* qfrag = reinterpret_cast<uint32_t*>(smem + (size_t)a.n_stage * stage_bytes);  // [ncw][2][TPW][4][2]
  float4* qpre = reinterpret_cast<float4*>(qfrag + ncw * 2 * TPW * 4 * 2);  // [ncw][TPW / 8][32 lanes]
  float* red = reinterpret_cast<float*>(qpre + ncw * 32 * (TPW / 8));  // [RM_SBUF][16 rows][RM_RED_STRIDE]
  StageMeta* meta = reinterpret_cast<StageMeta*>(red + RM_SBUF * 16 * RM_RED_STRIDE);
  GroupRec* grec = reinterpret_cast<GroupRec*>(meta + a.n_stage);                 // [RM_SBUF]
  uint32_t* pfrag = reinterpret_cast<uint32_t*>(grec + RM_SBUF);                  // [RM_SBUF][4 lanes][4]
  float* psc = reinterpret_cast<float*>(pfrag + RM_SBUF * 16);                    // [RM_SBUF] rescale factors
  uint64_t* full = reinterpret_cast<uint64_t*>(psc + RM_SBUF);
  uint64_t* empty = full + a.n_stage;
  uint64_t* sbar = empty + a.n_stage;  // [RM_SBUF] partial scores of a group are complete
  uint64_t* pbar = sbar + RM_SBUF;     // [RM_SBUF] the group's P fragments are published
  volatile int* abort_flag = reinterpret_cast<volatile int*>(pbar + RM_SBUF);
  int* plan = const_cast<int*>(reinterpret_cast<volatile int*>(abort_flag) + 4);  // [plan_pairs + 1], in-kernel plan

  {
    uint4* z = reinterpret_cast<uint4*>(stages);
    const int n16 = a.n_stage * stage_bytes / 16;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) z[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();  // the zeros precede the bulk copies into the same bytes
    // score slots of warps >= ncw are never written: they stay 0 for the vector sum
    for (int i = threadIdx.x; i < RM_SBUF * 16 * RM_RED_STRIDE; i += blockDim.x) red[i] = 0.f;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.n_stage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], ncw);
    }
    for (int i = 0; i < RM_SBUF; ++i) {
      mbar_init(&sbar[i], ncw);
      mbar_init(&pbar[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Under programmatic dependent launch everything above (shared memory only) overlaps the kernel before; the
  // routing outputs (idx, wk) and q are read only after the wait. The trigger lets the merge be scheduled.
  pdl_wait();
  pdl_trigger();

  // work units: every item in order, or (sparse plan) the items that hold rows: listed by read_compact_kernel, or
  // counted and scanned here by the whole block
  int64_t n_work = a.n_items;
  if (a.plan_pairs > 0) {
    const int np = a.plan_pairs;
    for (int pr = threadIdx.x; pr < np; pr += blockDim.x) plan[pr + 1] = pair_pieces(a, pr);
    __syncthreads();
    if (warp == 0) {  // lane l scans pairs [l * per, (l + 1) * per), then a warp scan of the lanes' sums
      const int per = (np + 31) / 32, b0 = min(np, lane * per), b1 = min(np, b0 + per);
      int sum = 0;
      for (int i = b0; i < b1; ++i) sum += plan[i + 1];
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int run = incl - sum;
      for (int i = b0; i < b1; ++i) {
        run += plan[i + 1];
        plan[i + 1] = run;
      }
      if (lane == 0) plan[0] = 0;
    }
    __syncthreads();
    n_work = plan[np];
  }
  // the producer's first 32 items are looked up together (one per lane), so their lookups overlap one another
  ItemRange mine;
  mine.active = false;
  mine.r0 = mine.r1 = 0;
  mine.base = nullptr;
  mine.row = 0;
  if (warp == 0) {
    if (a.item_list) n_work = *a.n_active;
    const int64_t my_w = blockIdx.x + (int64_t)lane * gridDim.x;
    if (my_w < n_work) mine = decode_item(a, work_item(a, plan, my_w));
  }
  __syncthreads();

  // ------------------------------------------------------------------------------------------- producer
  if (warp == 0) {
    // the whole warp walks the items in step; lane 0 owns the barriers and descriptors, and a stage's row
    // copies are issued by the lanes in parallel (row r by lane r % 32)
    const uint64_t pol = policy_evict_first();
    uint32_t it_count = 0;
    bool ok = true;
    // the CTA's items are decoded 32 at a time, one per lane (their page and row-range lookups overlap), and
    // handed to the whole warp by shuffles
    int64_t batch = 0;
    int64_t k_item = 0;  // this CTA's k-th item is blockIdx.x + k * gridDim.x
    for (int64_t wu = blockIdx.x; wu < n_work && ok; wu += gridDim.x, ++k_item) {
      const int64_t item = work_item(a, plan, wu);
      if ((k_item >> 5) != batch) {
        batch = k_item >> 5;
        const int64_t my_w = blockIdx.x + ((batch << 5) + lane) * (int64_t)gridDim.x;
        mine.active = false;
        mine.r0 = mine.r1 = 0;
        mine.base = nullptr;
        mine.row = 0;
        if (my_w < n_work) mine = decode_item(a, work_item(a, plan, my_w));
      }
      const int who = (int)(k_item & 31);  // the lane that decoded this item
      ItemRange it;
      it.active = __shfl_sync(0xffffffffu, (int)mine.active, who) != 0;
      it.r0 = __shfl_sync(0xffffffffu, mine.r0, who);
      it.r1 = __shfl_sync(0xffffffffu, mine.r1, who);
      it.row = __shfl_sync(0xffffffffu, (long long)mine.row, who);
      // the next item's row, from the lane that decoded it (the batch's last item leaves it to a global load)
      const long long nrow = __shfl_sync(0xffffffffu, mine.active ? (long long)mine.row : -1ll, (who + 1) & 31);
      it.base = reinterpret_cast<const char*>(
          __shfl_sync(0xffffffffu, (unsigned long long)reinterpret_cast<uintptr_t>(mine.base), who));
      if (!it.active || it.r1 <= it.r0) continue;
      for (int rs = it.r0; rs < it.r1 && ok; rs += a.rps) {
        const int nr = min(a.rps, it.r1 - rs);
        const bool last = rs + nr >= it.r1;
        // the group's key rows, then (untied values) the same rows of the value pool as a second stage
        for (int part = 0; part < (a.vslots ? 2 : 1); ++part) {
          const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
          bool good = true;
          if (lane == 0 && use > 0) good = mbar_wait_spin(&empty[slot], (use - 1) & 1);
          if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
          if (lane == 0) {
            meta[slot].item = item;
            meta[slot].nr = nr;
            meta[slot].row = it.row;
            meta[slot].next_row = who < 31 ? nrow : -1;
            meta[slot].flags = part == 0 ? ((rs == it.r0 ? RM_FIRST : 0) | (last && !a.vslots ? RM_LAST : 0))
                                         : (RM_VAL | (last ? RM_LAST : 0));
            mbar_arrive_expect_tx(&full[slot], (uint32_t)nr * a.row_bytes);
          }
          __syncwarp();  // the expected bytes are registered before any of the stage's copies is issued
          unsigned char* dst = stages + (size_t)slot * stage_bytes;
          const char* src = (part == 0 ? it.base : a.vslots + (it.base - a.slots)) + (int64_t)rs * a.row_bytes;
          for (int r = lane; r < nr; r += 32)
            bulk_g2s(dst + (size_t)r * row_stride, src + (int64_t)r * a.row_bytes, (uint32_t)a.row_bytes, &full[slot],
                     pol);
          ++it_count;
        }
      }
    }
    if (lane != 0) return;
    if (ok) {  // end-of-work descriptor
      const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
      if (use == 0 || mbar_wait_bounded(&empty[slot], (use - 1) & 1)) {
        meta[slot].item = -1;
        meta[slot].nr = 0;
        meta[slot].row = 0;
        meta[slot].next_row = -1;
        meta[slot].flags = RM_DONE;
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

  // ------------------------------------------------------------------------------------------- softmax warp
  // Tied reads only (untied reads keep the per-warp softmax of the value-stage loop below). Per posted group:
  // the 16 row scores from the consumers' partials, the online softmax of the current item (m, l per row lane),
  // P rounded to the slot type and packed as the MMA's B fragment, the rescale factor of the running sums;
  // then one arrive on the group's P barrier. At an item's last group it writes the item's (m, l).
  if (warp == ncw + 1) {
    if (a.vslots) return;
    const int prow = lane & 15;
    const int ka = (lane & 3) * 2;
    float m = -CUDART_INF_F, l = 0.f;
    for (uint32_t gs = 0;; ++gs) {
      const uint32_t b = gs % RM_SBUF;
      if (!mbar_wait_spin(&sbar[b], (gs / RM_SBUF) & 1) || *abort_flag) { *abort_flag = 1; return; }
      const GroupRec gr = grec[b];
      if (gr.flags & RM_DONE) return;
      if (gr.flags & RM_FIRST) { m = -CUDART_INF_F; l = 0.f; }
      // the row's partials are contiguous: four 16-byte loads (rows 80 bytes apart: conflict-free), a tree sum
      const float4* rr = reinterpret_cast<const float4*>(red + b * 16 * RM_RED_STRIDE + prow * RM_RED_STRIDE);
      float4 v4[RM_MAX_WARPS / 4];
#pragma unroll
      for (int j = 0; j < RM_MAX_WARPS / 4; ++j) v4[j] = 4 * j < ncw ? rr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      const float srow = ((v4[0].x + v4[0].y) + (v4[0].z + v4[0].w)) + ((v4[1].x + v4[1].y) + (v4[1].z + v4[1].w)) +
                         (((v4[2].x + v4[2].y) + (v4[2].z + v4[2].w)) + ((v4[3].x + v4[3].y) + (v4[3].z + v4[3].w)));
      const bool valid = prow < gr.gv;
      float p, sc = 1.f;
      if (SOFTMAX) {
        float mx = valid ? srow : -CUDART_INF_F;
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        const float m_new = fmaxf(m, mx);
        if (m_new != m) {
          sc = m == -CUDART_INF_F ? 0.f : exp2f(m - m_new);
          l *= sc;
          m = m_new;
        }
        p = valid ? exp2f(srow - m) : 0.f;
      } else {
        p = valid ? srow : 0.f;
      }
      // round p to the slot type (+ residual for bf16); l sums the values the MMA uses (per row lane)
      const T ph = from_f32<T>(p);
      const float phf = to_f32(ph);
      const T pl = from_f32<T>(SPLIT ? p - phf : 0.f);
      if (SOFTMAX && lane < 16) l += phf + (SPLIT ? to_f32(pl) : 0.f);
      uint16_t uh, ul;
      memcpy(&uh, &ph, 2);
      memcpy(&ul, &pl, 2);
      const uint32_t ubits = (uint32_t)uh | ((uint32_t)ul << 16);
      const uint32_t e0 = __shfl_sync(0xffffffffu, ubits, ka);
      const uint32_t e1 = __shfl_sync(0xffffffffu, ubits, ka + 1);
      const uint32_t e8 = __shfl_sync(0xffffffffu, ubits, ka + 8);
      const uint32_t e9 = __shfl_sync(0xffffffffu, ubits, ka + 9);
      if (lane < 4) {
        uint4 f;
        f.x = (e0 & 0xffffu) | (e1 << 16);            // P rows 2l, 2l+1
        f.y = (e8 & 0xffffu) | (e9 << 16);            // P rows 2l+8, 2l+9
        f.z = (e0 >> 16) | (e1 & 0xffff0000u);        // residuals (bf16)
        f.w = (e8 >> 16) | (e9 & 0xffff0000u);
        reinterpret_cast<uint4*>(pfrag + b * 16)[lane] = f;
      }
      if (lane == 0) psc[b] = sc;
      __syncwarp();
      if (lane == 0) mbar_arrive(&pbar[b]);
      if (gr.flags & RM_LAST) {
        float lt = l;
        lt += __shfl_xor_sync(0xffffffffu, lt, 1);
        lt += __shfl_xor_sync(0xffffffffu, lt, 2);
        lt += __shfl_xor_sync(0xffffffffu, lt, 4);
        lt += __shfl_xor_sync(0xffffffffu, lt, 8);
        lt += __shfl_xor_sync(0xffffffffu, lt, 16);
        if (lane == 0) {
          a.part_ml[gr.item * 2] = SOFTMAX ? m : 0.f;
          a.part_ml[gr.item * 2 + 1] = SOFTMAX ? lt : 1.f;
        }
      }
    }
  }

  // ------------------------------------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int d0 = cw * (16 * TPW);
  const int nt = min(TPW, (a.d_s - d0) / 16);  // >= 1 (host: d_s % 16 == 0, ncw = ceil(d_s / (16 * TPW)))
  uint32_t* qf = qfrag + cw * 2 * TPW * 4 * 2;
  const uint32_t stages_u32 = smem_u32(stages);
  const int mtx = lane >> 3, r8 = lane & 7;
  const uint32_t off_s = (uint32_t)((r8 + (mtx & 1) * 8) * row_stride + (mtx >> 1) * 16 + d0 * 2);
  const uint32_t off_a = (uint32_t)((r8 + (mtx >> 1) * 8) * row_stride + (mtx & 1) * 16 + d0 * 2);
  const int prow = lane & 15;  // the group row this lane finishes
  const int ka = (lane & 3) * 2;

  float acc[TPW][4];
  float m = -CUDART_INF_F, l = 0.f;
  uint32_t it_count = 0, grp = 0;
  uint32_t vb0 = 0u, vb1 = 0u, vc0 = 0u, vc1 = 0u;  // P fragments of the last key group (untied values)
  auto write_partial = [&](int64_t item) {
    float* pa = a.part_acc + item * (int64_t)a.d_s;
    if ((lane & 3) == 0) {
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (t < nt) {
          const int d = d0 + t * 16 + (lane >> 2);
          pa[d] = acc[t][0];
          pa[d + 8] = acc[t][2];
        }
      }
    }
    if (cw == 0 && lane == 0) {
      a.part_ml[item * 2] = SOFTMAX ? m : 0.f;
      a.part_ml[item * 2 + 1] = SOFTMAX ? l : 1.f;
    }
  };

  // q fragments of an item (B operand, query in column 0 = lanes 0..3), hi and residual, into this warp's slot
  // q of the CTA's next item (its row comes with the item's first stage) is copied into this lane's slots of qpre
  // when an item starts (cp.async, no registers held), so the next item's first group finds it on chip
  float4* qp = qpre + cw * 32 * (TPW / 8);
  int64_t qnext_row = -1;
  auto load_q = [&](const StageMeta& md) {
    // the warp's 16*TPW columns of q: lane i loads columns [4i, 4i + 4) of each 128-column block with one
    // 16-byte load and writes them, packed to the slot type, into their B-fragment words (tile t = i / 4:
    // columns 16t + r; pairs r < 8 are the fragment's first word of lane r / 2, pairs r >= 8 its second)
    const int64_t row = md.row;
    const float* qr = a.q + row * a.d_s;
    float4 qv[TPW / 8];
    const bool pre = row == qnext_row;
    if (pre) cp_async_wait_all();  // this lane's own copies
#pragma unroll
    for (int u = 0; u < TPW / 8; ++u) {
      const int t = u * 8 + (lane >> 2);
      if (t < nt)
        qv[u] = pre ? qp[u * 32 + lane] : __ldg(reinterpret_cast<const float4*>(qr + d0 + t * 16 + (lane & 3) * 4));
    }
    qnext_row = md.next_row;
    if (qnext_row >= 0) {
      const float* nq = a.q + qnext_row * a.d_s;
#pragma unroll
      for (int u = 0; u < TPW / 8; ++u) {
        const int t = u * 8 + (lane >> 2);
        if (t < nt) cp_async16(qp + u * 32 + lane, nq + d0 + t * 16 + (lane & 3) * 4);
      }
    }
#pragma unroll
    for (int u = 0; u < TPW / 8; ++u) {
      const int t = u * 8 + (lane >> 2);  // tile of this lane's four columns
      if (t < nt) {
        const float4 v = qv[u];
        const int r0 = (lane & 3) * 4;  // column of v.x within the tile
        const int w = r0 < 8 ? 0 : 1;   // first or second fragment word
        const int l0 = (r0 & 7) >> 1;   // fragment lane of the pair (v.x, v.y); (v.z, v.w) goes to l0 + 1
        const float x0 = v.x * a.qscale, x1 = v.y * a.qscale, x2 = v.z * a.qscale, x3 = v.w * a.qscale;
        float h0, h1, h2, h3, e0, e1, e2, e3;
        qf[t * 8 + l0 * 2 + w] = pack2<T>(x0, x1, h0, h1);
        qf[t * 8 + (l0 + 1) * 2 + w] = pack2<T>(x2, x3, h2, h3);
        qf[(TPW + t) * 8 + l0 * 2 + w] = SPLIT ? pack2<T>(x0 - h0, x1 - h1, e0, e1) : 0u;
        qf[(TPW + t) * 8 + (l0 + 1) * 2 + w] = SPLIT ? pack2<T>(x2 - h2, x3 - h3, e2, e3) : 0u;
      }
    }
    __syncwarp();
  };

  if (!a.vslots) {
    // Tied K = V, pipelined by one 16-row group: post group g's partial scores, then accumulate group g - 1
    // with the P fragments the softmax warp published for it. RM_SBUF buffers: a consumer posts group g only
    // after it waited for the P of group g - 2, so the softmax warp is done reading buffer (g - 4) by then; the
    // softmax warp writes the P of group g after every consumer posted g, i.e. finished reading P of g - 1.
    struct Pend {
      uint32_t slot, gidx;
      int g0;
      bool first, last_group, last;
      long long item;
    };
    Pend pd{};
    bool have = false;
    uint32_t gseq = 0;
    auto post = [&](uint32_t slot, int g0, const StageMeta& md) {
      const uint32_t b = gseq % RM_SBUF;
      const uint32_t gbase = stages_u32 + slot * (uint32_t)stage_bytes + (uint32_t)(g0 * row_stride);
      float sa[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) sa[c][0] = sa[c][1] = sa[c][2] = sa[c][3] = 0.f;
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (t < nt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(gbase + off_s + t * 32, a0, a1, a2, a3);
          uint32_t b0 = 0u, b1 = 0u;
          if (lane < 4) {
            b0 = qf[t * 8 + lane * 2];
            b1 = qf[t * 8 + lane * 2 + 1];
          }
          mma16816<T>(sa[t & 3], a0, a1, a2, a3, b0, b1);
          if (SPLIT) {
            uint32_t c0 = 0u, c1 = 0u;
            if (lane < 4) {
              c0 = qf[(TPW + t) * 8 + lane * 2];
              c1 = qf[(TPW + t) * 8 + lane * 2 + 1];
            }
            mma16816<T>(sa[(t + 2) & 3], a0, a1, a2, a3, c0, c1);
          }
        }
      }
      const float sc_lo = (sa[0][0] + sa[1][0]) + (sa[2][0] + sa[3][0]);  // row lane/4 (lanes with lane%4 == 0)
      const float sc_hi = (sa[0][2] + sa[1][2]) + (sa[2][2] + sa[3][2]);  // row lane/4 + 8
      float* rb = red + b * 16 * RM_RED_STRIDE;
      if ((lane & 3) == 0) {
        rb[(lane >> 2) * RM_RED_STRIDE + cw] = sc_lo;
        rb[((lane >> 2) + 8) * RM_RED_STRIDE + cw] = sc_hi;
      }
      if (cw == 0 && lane == 0) {
        const bool last_group = g0 + 16 >= md.nr;
        GroupRec gr;
        gr.item = md.item;
        gr.flags = ((md.flags & RM_FIRST) && g0 == 0 ? RM_FIRST : 0) | (last_group && (md.flags & RM_LAST) ? RM_LAST : 0);
        gr.gv = min(16, md.nr - g0);
        grec[b] = gr;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sbar[b]);
    };
    auto post_done = [&]() {
      const uint32_t b = gseq % RM_SBUF;
      if (cw == 0 && lane == 0) {
        GroupRec gr;
        gr.item = -1;
        gr.flags = RM_DONE;
        gr.gv = 0;
        grec[b] = gr;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sbar[b]);
    };
    // accumulate a posted group with its published P; release the stage after its last group
    auto finish = [&](const Pend& g) -> bool {
      const uint32_t b = g.gidx % RM_SBUF;
      if (!mbar_wait_spin(&pbar[b], (g.gidx / RM_SBUF) & 1) || *abort_flag) {
        *abort_flag = 1;
        return false;
      }
      if (g.first) {
#pragma unroll
        for (int t = 0; t < TPW; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
      }
      const float sc = psc[b];
      if (sc != 1.f) {
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          acc[t][0] *= sc;
          acc[t][2] *= sc;
        }
      }
      uint4 f = make_uint4(0u, 0u, 0u, 0u);
      if (lane < 4) f = reinterpret_cast<const uint4*>(pfrag + b * 16)[lane];
      const uint32_t gbase = stages_u32 + g.slot * (uint32_t)stage_bytes + (uint32_t)(g.g0 * row_stride);
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (t < nt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(gbase + off_a + t * 32, a0, a1, a2, a3);
          mma16816<T>(acc[t], a0, a1, a2, a3, f.x, f.y);
          if (SPLIT) mma16816<T>(acc[t], a0, a1, a2, a3, f.z, f.w);
        }
      }
      if (g.last_group) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[g.slot]);
        if (g.last) {  // this warp's columns of the item's partial (the softmax warp writes its m, l)
          float* pa = a.part_acc + g.item * (int64_t)a.d_s;
          if ((lane & 3) == 0) {
#pragma unroll
            for (int t = 0; t < TPW; ++t) {
              if (t < nt) {
                const int d = d0 + t * 16 + (lane >> 2);
                pa[d] = acc[t][0];
                pa[d + 8] = acc[t][2];
              }
            }
          }
        }
      }
      return true;
    };

    bool ok = true;
    while (ok) {
      const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
      ++it_count;
      if (!mbar_wait_spin(&full[slot], use & 1) || *abort_flag) { *abort_flag = 1; ok = false; break; }
      const StageMeta md = meta[slot];
      if (md.flags & RM_DONE) {
        post_done();
        break;
      }
      if (md.flags & RM_FIRST) load_q(md);
      for (int g0 = 0; g0 < md.nr; g0 += 16) {
        post(slot, g0, md);
        if (have && !finish(pd)) { ok = false; break; }
        pd.slot = slot;
        pd.gidx = gseq;
        pd.g0 = g0;
        pd.first = (md.flags & RM_FIRST) && g0 == 0;
        pd.last_group = g0 + 16 >= md.nr;
        pd.last = pd.last_group && (md.flags & RM_LAST);
        pd.item = md.item;
        have = true;
        ++gseq;
      }
    }
    if (ok && have) finish(pd);
    return;
  }

  while (true) {
    const uint32_t slot = it_count % a.n_stage, use = it_count / a.n_stage;
    ++it_count;
    if (!mbar_wait_bounded(&full[slot], use & 1) || *abort_flag) { *abort_flag = 1; break; }
    const StageMeta md = meta[slot];
    if (md.flags & RM_DONE) break;

    if (md.flags & RM_VAL) {
      // untied values: the group's P (kept from its key stage) times these value rows
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
      if (md.flags & RM_LAST) write_partial(md.item);
      continue;
    }

    if (md.flags & RM_FIRST) {
      // q fragments (B operand, query in column 0 = lanes 0..3), hi and residual, into this warp's slot
      if (lane < 4) {
        const int64_t row = (md.item / a.n_split) / a.k;
        const float* qr = a.q + row * a.d_s;
        for (int t = 0; t < nt; ++t) {
          const int k = d0 + t * 16 + lane * 2;
          const float x0 = __ldg(qr + k) * a.qscale, x1 = __ldg(qr + k + 1) * a.qscale;
          const float x2 = __ldg(qr + k + 8) * a.qscale, x3 = __ldg(qr + k + 9) * a.qscale;
          float h0, h1, h2, h3, l0, l1, l2, l3;
          qf[t * 8 + lane * 2] = pack2<T>(x0, x1, h0, h1);
          qf[t * 8 + lane * 2 + 1] = pack2<T>(x2, x3, h2, h3);
          qf[(TPW + t) * 8 + lane * 2] = SPLIT ? pack2<T>(x0 - h0, x1 - h1, l0, l1) : 0u;
          qf[(TPW + t) * 8 + lane * 2 + 1] = SPLIT ? pack2<T>(x2 - h2, x3 - h3, l2, l3) : 0u;
        }
      }
      __syncwarp();
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
      // ---- scores: four accumulator chains
      float sa[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) sa[c][0] = sa[c][1] = sa[c][2] = sa[c][3] = 0.f;
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (t < nt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(gbase + off_s + t * 32, a0, a1, a2, a3);
          uint32_t b0 = 0u, b1 = 0u;
          if (lane < 4) {
            b0 = qf[t * 8 + lane * 2];
            b1 = qf[t * 8 + lane * 2 + 1];
          }
          mma16816<T>(sa[t & 3], a0, a1, a2, a3, b0, b1);
          if (SPLIT) {
            uint32_t c0 = 0u, c1 = 0u;
            if (lane < 4) {
              c0 = qf[(TPW + t) * 8 + lane * 2];
              c1 = qf[(TPW + t) * 8 + lane * 2 + 1];
            }
            mma16816<T>(sa[(t + 2) & 3], a0, a1, a2, a3, c0, c1);
          }
        }
      }
      const float sc_lo = (sa[0][0] + sa[1][0]) + (sa[2][0] + sa[3][0]);  // row lane/4 (lanes with lane%4 == 0)
      const float sc_hi = (sa[0][2] + sa[1][2]) + (sa[2][2] + sa[3][2]);  // row lane/4 + 8
      float srow;
      if (ncw > 1) {
        const int b = grp & 1;
        float* rb = red + b * 16 * RM_RED_STRIDE;
        if ((lane & 3) == 0) {
          rb[(lane >> 2) * RM_RED_STRIDE + cw] = sc_lo;
          rb[((lane >> 2) + 8) * RM_RED_STRIDE + cw] = sc_hi;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sbar[b]);
        if (!mbar_wait_bounded(&sbar[b], (grp >> 1) & 1) || *abort_flag) {
          *abort_flag = 1;
          aborted = true;
          break;
        }
        srow = 0.f;
        // the row's partials are contiguous: four 16-byte loads (rows 80 bytes apart: conflict-free), a tree sum
        const float4* rr = reinterpret_cast<const float4*>(rb + prow * RM_RED_STRIDE);
        float4 v4[RM_MAX_WARPS / 4];
#pragma unroll
        for (int j = 0; j < RM_MAX_WARPS / 4; ++j) v4[j] = 4 * j < ncw ? rr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        srow = ((v4[0].x + v4[0].y) + (v4[0].z + v4[0].w)) + ((v4[1].x + v4[1].y) + (v4[1].z + v4[1].w)) +
               (((v4[2].x + v4[2].y) + (v4[2].z + v4[2].w)) + ((v4[3].x + v4[3].y) + (v4[3].z + v4[3].w)));
      } else {
        const float v_lo = __shfl_sync(0xffffffffu, sc_lo, (prow & 7) * 4);
        const float v_hi = __shfl_sync(0xffffffffu, sc_hi, (prow & 7) * 4);
        srow = prow < 8 ? v_lo : v_hi;
      }
      ++grp;
      const bool valid = prow < gv;
      float p;
      if (SOFTMAX) {
        float mx = valid ? srow : -CUDART_INF_F;
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        const float m_new = fmaxf(m, mx);
        if (m_new != m) {
          const float sc = exp2f(m - m_new);
          l *= sc;
#pragma unroll
          for (int t = 0; t < TPW; ++t) {
            acc[t][0] *= sc;
            acc[t][2] *= sc;
          }
          m = m_new;
        }
        p = valid ? exp2f(srow - m) : 0.f;
      } else {
        p = valid ? srow : 0.f;
      }
      // round p to the slot type (+ residual for bf16); l sums the values the MMA uses
      const T ph = from_f32<T>(p);
      const float phf = to_f32(ph);
      const T pl = from_f32<T>(SPLIT ? p - phf : 0.f);
      if (SOFTMAX) {
        float ps = phf + (SPLIT ? to_f32(pl) : 0.f);
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        ps += __shfl_xor_sync(0xffffffffu, ps, 8);
        l += ps;
      }
      uint16_t uh, ul;
      memcpy(&uh, &ph, 2);
      memcpy(&ul, &pl, 2);
      const uint32_t ubits = (uint32_t)uh | ((uint32_t)ul << 16);
      const uint32_t e0 = __shfl_sync(0xffffffffu, ubits, ka);
      const uint32_t e1 = __shfl_sync(0xffffffffu, ubits, ka + 1);
      const uint32_t e8 = __shfl_sync(0xffffffffu, ubits, ka + 8);
      const uint32_t e9 = __shfl_sync(0xffffffffu, ubits, ka + 9);
      const uint32_t pb0 = lane < 4 ? ((e0 & 0xffffu) | (e1 << 16)) : 0u;
      const uint32_t pb1 = lane < 4 ? ((e8 & 0xffffu) | (e9 << 16)) : 0u;
      const uint32_t pc0 = lane < 4 ? ((e0 >> 16) | (e1 & 0xffff0000u)) : 0u;
      const uint32_t pc1 = lane < 4 ? ((e8 >> 16) | (e9 & 0xffff0000u)) : 0u;
      if (a.vslots) {  // untied: the value stage that follows does the accumulation (one group per stage)
        vb0 = pb0; vb1 = pb1; vc0 = pc0; vc1 = pc1;
        continue;
      }
      // ---- accumulate: acc[d, 0] += sum_rows K[row, d] p[row]
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
    if (md.flags & RM_LAST) write_partial(md.item);
  }
}

}  // namespace xencb

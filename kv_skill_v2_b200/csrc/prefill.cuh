// Prefill (registration) read on the 5th-generation tensor cores: the dense read of LibraryInjector._branch
// (xenc/injector.py:239-265) for T query tokens per Library, as two tcgen05 GEMMs (kind::f16, f32 accumulate
// in TMEM, operands staged by 2-D TMA with 64-byte (scores) or 128-byte (read) swizzle, no multicast):
//
//   scores  S[t, c, j] = q16[t] . K[c, j]                                   CTA tile: 128 tokens x one chunk
//           P[t, c, j] = w[t, c] * softmax_j<n_c(read_temp * S[t, c, :])_j   (softmax read)
//                      = w[t, c] * S[t, c, j] / sqrt(n_c)                    (linear read)
//                      = 0 for j >= n_c                                      P stored f16 [R, C * ncol]
//   read    r[t]       = sum_{c, j} P[t, c, j] K[c, j]                       CTA tile: 128 tokens x 256 of d_s
//
// The chunk softmax is complete inside one scores tile (a chunk's <= 512 scores of a token sit in one TMEM row),
// so P carries the final two-level weights and the read is a plain GEMM over all slots. In the read the slots
// are the contraction dimension while a slot row stores d_s contiguously, so K enters as an MN-major B operand.
// q is rounded to f16 for the first product (the slots are f16 already); P is f16 in [0, w].
// Warp roles: warp 0 lane 0 issues TMA, warp 1 lane 0 issues tcgen05.mma; the epilogue runs on 16 warps in the
// scores kernel (warp w reads TMEM lane quarter w % 4 = 32 token rows, column group (w - 2) / 4 = 128 columns;
// the four groups of a row combine their (max, sum) in shared memory) and on 4 warps in the read kernel
// (thread = token row = TMEM lane). Every wait is bounded; TMEM is freed on every path.
#pragma once

#include <math_constants.h>

#include "tc.cuh"

namespace xencb {

// 2^x for the chunk softmax of the scores epilogue: the PTX ISA's ex2.approx.ftz.f32 instruction (relative error
// about 2^-22 over the range used here, denormal results flushed to 0). The values end as f16 P (11 significant
// bits, smallest subnormal 2^-24), so neither the approximation nor the flush shows in P; the exponent is formed as
// one FMA, x * qscale - max * qscale. Measured on config 3: scores + read kernels 9.54 -> 9.28 ms against exp2f.
__device__ __forceinline__ float pf_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
#define PF_EXP2(x) pf_exp2(x)

constexpr int PF_BM = 128;      // tokens per CTA (UMMA M)
constexpr int PF_BK = 64;       // f16 per 128-byte swizzle row = one k-block
constexpr int PF_THREADS = 192;         // read kernel: producer, MMA, 4 epilogue warps
constexpr int PF_S_EPI_WARPS = 16;      // scores: 4 column groups x 4 TMEM lane quarters
constexpr int PF_S_THREADS = 32 * (2 + PF_S_EPI_WARPS);
constexpr int PF_S_BK = 32;     // scores k-block: 32 f16 = 64-byte swizzle rows
constexpr int PF_S_STAGES = 5;  // scores: A 8 KB + B up to 32 KB per stage
constexpr int PF_S_BBYTES = 512 * 64;
constexpr int PF_S_STAGE = PF_BM * 64 + PF_S_BBYTES;
constexpr size_t PF_S_SMEM = 1024 + (size_t)PF_S_STAGES * PF_S_STAGE + 256 + 4 * 128 * 2 * 4;
constexpr int PF_R_STAGES = 4;  // read: A 16 KB + B 4 x 8 KB per stage
constexpr int PF_R_BN = 256;    // columns of d_s per read CTA
constexpr int PF_R_STAGE = PF_BM * 128 + (PF_R_BN / 64) * 64 * 128;
constexpr size_t PF_R_SMEM = 1024 + (size_t)PF_R_STAGES * PF_R_STAGE + 256;

struct PrefillArgs {
  int64_t n_rows;          // R
  int64_t rows_per_lib;    // T
  int d_s;
  int n_chunks;            // C (page-table width)
  int page_rows;           // N
  int ncol;                // round_up(N, 64): P columns per chunk, <= 512
  int64_t n_pages;
  const int32_t* page_of;      // [n_lib, C]
  const int32_t* n_valid;      // [n_lib, C]
  const int32_t* n_chunks_of;  // [n_lib] or null
  const float* w;              // [R, C]
  float qscale;                // read_temp * log2(e)
  int softmax;
  __half* P;                   // [R, C * ncol]
  float* r_out;                // [R, d_s]
};

struct PfBars {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* done;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

__device__ __forceinline__ PfBars pf_bars(unsigned char* after_stages, int n_stage) {
  PfBars b;
  b.full = reinterpret_cast<uint64_t*>(after_stages);
  b.empty = b.full + n_stage;
  b.done = b.empty + n_stage;
  b.tmem_slot = reinterpret_cast<uint32_t*>(b.done + 1);
  b.abort_flag = reinterpret_cast<volatile int*>(b.tmem_slot + 1);
  return b;
}

__device__ __forceinline__ void pf_setup(const PfBars& b, int n_stage, uint32_t tmem_cols) {
  const int warp = threadIdx.x >> 5;
  if (warp == 1) {
    tc_alloc(b.tmem_slot, tmem_cols);
    tc_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < n_stage; ++i) {
      mbar_init(&b.full[i], 1);
      mbar_init(&b.empty[i], 1);
    }
    mbar_init(b.done, 1);
    *b.abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// ---------------------------------------------------------------------------------------------------- scores
// The scores epilogue of one CTA (16 warps, warps 2..17): token row rr of the tile (TMEM lane), columns
// [128 cg, 128 cg + 128): the chunk softmax, the routing weight, f16 P.
// A tile whose 128 rows all belong to the Library stages P in shared memory (the operand stages, free once the
// MMAs are done) as ncol / 64 boxes of [128 rows][64 columns] f16 in the 128-byte swizzle (16-byte chunk j of row
// r at chunk j ^ (r % 8): conflict-free for the row-per-thread writes) and writes them with TMA stores, one
// coalesced box each; a partial tile stores its valid rows directly.
__device__ __forceinline__ void pf_scores_epilogue(const PrefillArgs& a, const PfBars& bars, uint32_t taddr, int warp,
                                                   int lane, int64_t lib, int c, int64_t t0, int64_t row0,
                                                   bool page_ok, const CUtensorMap* map_p, unsigned char* tile) {
  float* part = reinterpret_cast<float*>(const_cast<int*>(bars.abort_flag) + 4);  // [4][128 rows][2] (max, sum)
  const int q4 = warp & 3, cg = (warp - 2) >> 2;
  const int rr = q4 * 32 + lane;
  const int64_t t = row0 + rr;
  const bool row_ok = t0 + rr < a.rows_per_lib && t < a.n_rows;
  const int nc = a.n_chunks_of ? min(a.n_chunks_of[lib], a.n_chunks) : a.n_chunks;
  int nv = a.n_valid[lib * a.n_chunks + c];
  if (nv > a.page_rows) {
    nv = a.page_rows;
    if (threadIdx.x == 64) flag_error(XENCB_DEV_CLAMPED);
  }
  if (!page_ok) {
    nv = 0;
    if (threadIdx.x == 64) flag_error(XENCB_DEV_BADPAGE);
  }
  if (nv < 0 || c >= nc) nv = 0;
  const float wt = row_ok ? a.w[t * a.n_chunks + c] : 0.f;
  const bool ok = mbar_wait_bounded(bars.done, 0) && !*bars.abort_flag;
  tc_fence_after();
  const uint32_t tl = taddr + ((uint32_t)(q4 * 32) << 16);
  const int cbeg = cg * 128, cend = min(a.ncol, cbeg + 128);
  float m = -CUDART_INF_F, l = 0.f;
  if (a.softmax) {
    // pass 1: this group's (max, sum) by the online rule over 32-column loads; blocks that are all valid skip the
    // per-column test, exponents as one FMA (x * qscale - max * qscale), two running sums
    for (int c0 = cbeg; c0 < cend; c0 += 32) {
      float v[32];
      tc_ld32(tl + (uint32_t)c0, v);
      const bool full = c0 + 32 <= nv;
      float mx = -CUDART_INF_F;
      if (full) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < nv) mx = fmaxf(mx, v[i]);
      }
      const float mn = fmaxf(m, mx);
      if (mn != -CUDART_INF_F) {
        const float mq = mn * a.qscale;
        float s0 = 0.f, s1 = 0.f;
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            s0 += PF_EXP2(fmaf(v[i], a.qscale, -mq));
            s1 += PF_EXP2(fmaf(v[i + 1], a.qscale, -mq));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c0 + i < nv) s0 += PF_EXP2(fmaf(v[i], a.qscale, -mq));
        }
        l = (m == -CUDART_INF_F ? 0.f : l * PF_EXP2((m - mn) * a.qscale)) + (s0 + s1);
        m = mn;
      }
    }
    part[(cg * 128 + rr) * 2] = m;
    part[(cg * 128 + rr) * 2 + 1] = l;
    named_bar_sync(1, 32 * PF_S_EPI_WARPS);
    float M = -CUDART_INF_F;
#pragma unroll
    for (int g = 0; g < 4; ++g) M = fmaxf(M, part[(g * 128 + rr) * 2]);
    float L = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float mg = part[(g * 128 + rr) * 2], lg = part[(g * 128 + rr) * 2 + 1];
      if (lg > 0.f) L += lg * exp2f((mg - M) * a.qscale);
    }
    m = M;
    l = L;
  }
  const float coef = (!ok || nv == 0 || wt == 0.f) ? 0.f : (a.softmax ? wt / l : wt * rsqrtf((float)nv));
  __half* prow = a.P + t * ((int64_t)a.n_chunks * a.ncol) + (int64_t)c * a.ncol;
  const bool via_tma = t0 + PF_BM <= a.rows_per_lib && row0 + PF_BM <= a.n_rows;  // the same for the whole CTA
  const float mq = m * a.qscale;
  // pass 2: P for this group's columns
  for (int c0 = cbeg; c0 < cend; c0 += 32) {
    float v[32];
    tc_ld32(tl + (uint32_t)c0, v);
    uint4* dst = reinterpret_cast<uint4*>(prow + c0);
    const bool full = coef != 0.f && c0 + 32 <= nv;
#pragma unroll
    for (int i8 = 0; i8 < 32; i8 += 8) {  // 8 values -> one 16-byte store
      uint32_t pk[4];
#pragma unroll
      for (int i = i8; i < i8 + 8; i += 2) {
        float x0 = 0.f, x1 = 0.f;
        if (full) {
          x0 = a.softmax ? coef * PF_EXP2(fmaf(v[i], a.qscale, -mq)) : coef * v[i];
          x1 = a.softmax ? coef * PF_EXP2(fmaf(v[i + 1], a.qscale, -mq)) : coef * v[i + 1];
        } else if (coef != 0.f) {
          if (c0 + i < nv) x0 = a.softmax ? coef * PF_EXP2(fmaf(v[i], a.qscale, -mq)) : coef * v[i];
          if (c0 + i + 1 < nv) x1 = a.softmax ? coef * PF_EXP2(fmaf(v[i + 1], a.qscale, -mq)) : coef * v[i + 1];
        }
        float r0, r1;
        pk[(i - i8) / 2] = pack2<__half>(x0, x1, r0, r1);
      }
      if (via_tma) {
        const int col = c0 + i8, box = col >> 6, ch = (col & 63) >> 3;
        *reinterpret_cast<uint4*>(tile + box * (PF_BM * 128) + rr * 128 + ((ch ^ (rr & 7)) << 4)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      } else if (row_ok) {
        dst[i8 / 8] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
  }
  if (via_tma) {
    fence_proxy_async_smem();  // the generic-proxy writes above, before the TMA reads them
    named_bar_sync(1, 32 * PF_S_EPI_WARPS);
    if (warp == 2 && lane == 0) {
      for (int b = 0; b < a.ncol / 64; ++b)
        tma_store_2d(map_p, tile + b * (PF_BM * 128), c * a.ncol + b * 64, (int)row0);
      bulk_commit();
      bulk_wait_read0();  // the shared memory stays in place until the stores have read it
    }
  }
}

__global__ void __launch_bounds__(PF_S_THREADS, 1) prefill_scores_kernel(const __grid_constant__ CUtensorMap map_q,
                                                                       const __grid_constant__ CUtensorMap map_k,
                                                                       const __grid_constant__ CUtensorMap map_p,
                                                                       const PrefillArgs a, int b_box_rows) {
  extern __shared__ unsigned char pf_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~uintptr_t(1023));
  const PfBars bars = pf_bars(smem + PF_S_STAGES * PF_S_STAGE, PF_S_STAGES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t lib = blockIdx.z;
  const int c = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.x * PF_BM;       // token offset inside the Library
  const int64_t row0 = lib * a.rows_per_lib + t0;        // first q row of the tile
  const int nkb = a.d_s / PF_S_BK;
  const int nb = (a.ncol + b_box_rows - 1) / b_box_rows;  // B boxes per stage (1 or 2)
  const uint32_t tx = (uint32_t)(PF_BM * 64 + nb * b_box_rows * 64);
  int64_t page = a.page_of[lib * a.n_chunks + c];
  const bool page_ok = page >= 0 && page < a.n_pages;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_q);
    prefetch_tensormap(&map_k);
  }
  pf_setup(bars, PF_S_STAGES, 512);
  const uint32_t taddr = *bars.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t stream = policy_evict_first();
      // a bad page is never read: its coordinates are moved past the pool (TMA fills zeros there)
      const int ybase = page_ok ? (int)(page * a.page_rows) : (int)(a.n_pages * a.page_rows);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % PF_S_STAGES, use = kb / PF_S_STAGES;
        if (use > 0 && (!mbar_wait_bounded(&bars.empty[s], (use - 1) & 1) || *bars.abort_flag)) {
          *bars.abort_flag = 1;
          break;
        }
        unsigned char* st = smem + s * PF_S_STAGE;
        mbar_arrive_expect_tx(&bars.full[s], tx);
        tma_load_2d(st, &map_q, kb * PF_S_BK, (int)row0, &bars.full[s]);
        for (int i = 0; i < nb; ++i)
          tma_load_2d_hint(st + PF_BM * 64 + i * b_box_rows * 64, &map_k, kb * PF_S_BK, ybase + i * b_box_rows,
                           &bars.full[s], stream);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const int n_0 = a.ncol < 256 ? a.ncol : 256, n_1 = a.ncol - n_0;
      const uint32_t id0 = umma_idesc(UMMA_F16, UMMA_F16, PF_BM, n_0);
      const uint32_t id1 = umma_idesc(UMMA_F16, UMMA_F16, PF_BM, n_1 > 0 ? n_1 : 16);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % PF_S_STAGES, use = kb / PF_S_STAGES;
        if (!mbar_wait_bounded(&bars.full[s], use & 1) || *bars.abort_flag) { *bars.abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * PF_S_STAGE);
        const uint32_t bq = st + PF_BM * 64;
#pragma unroll
        for (int ks = 0; ks < PF_S_BK / 16; ++ks) {  // 16 f16 = 32 bytes per UMMA k-step
          const uint64_t ad = umma_desc_k_sw64(st + ks * 32);
          tc_mma<0>(taddr, ad, umma_desc_k_sw64(bq + ks * 32), id0, kb > 0 || ks > 0);
          if (n_1 > 0) tc_mma<0>(taddr + 256u, ad, umma_desc_k_sw64(bq + 256 * 64 + ks * 32), id1, kb > 0 || ks > 0);
        }
        tc_commit(&bars.empty[s]);
      }
      tc_commit(bars.done);
    }
  } else {
    pf_scores_epilogue(a, bars, taddr, warp, lane, lib, c, t0, row0, page_ok, &map_p, smem);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tc_dealloc(taddr, 512);
}

// ---------------------------------------------------------------------------------------------------- read
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_read_kernel(const __grid_constant__ CUtensorMap map_p,
                                                                     const __grid_constant__ CUtensorMap map_k,
                                                                     const PrefillArgs a) {
  extern __shared__ unsigned char pf_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~uintptr_t(1023));
  const PfBars bars = pf_bars(smem + PF_R_STAGES * PF_R_STAGE, PF_R_STAGES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t lib = blockIdx.z;
  const int n0 = blockIdx.y * PF_R_BN;
  const int nt = min(PF_R_BN, a.d_s - n0);  // columns of this CTA (a multiple of 64)
  const int nbox = nt / 64;
  const int64_t t0 = (int64_t)blockIdx.x * PF_BM;
  const int64_t row0 = lib * a.rows_per_lib + t0;
  const int nc = a.n_chunks_of ? min(a.n_chunks_of[lib], a.n_chunks) : a.n_chunks;
  const int kpc = a.ncol / PF_BK;  // k-blocks per chunk
  const int nkb = nc * kpc;
  const uint32_t tx = (uint32_t)(PF_BM * 128 + nbox * 64 * 128);

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_p);
    prefetch_tensormap(&map_k);
  }
  pf_setup(bars, PF_R_STAGES, 256);
  const uint32_t taddr = *bars.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t stream = policy_evict_first();
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % PF_R_STAGES, use = kb / PF_R_STAGES;
        if (use > 0 && (!mbar_wait_bounded(&bars.empty[s], (use - 1) & 1) || *bars.abort_flag)) {
          *bars.abort_flag = 1;
          break;
        }
        const int c = kb / kpc, jb = kb - c * kpc;
        const int64_t page = a.page_of[lib * a.n_chunks + c];
        // P is 0 for a bad page (the scores kernel flagged it); its rows are read from past the pool (zeros)
        const int y = (page >= 0 && page < a.n_pages ? (int)(page * a.page_rows) : (int)(a.n_pages * a.page_rows)) +
                      jb * PF_BK;
        unsigned char* st = smem + s * PF_R_STAGE;
        mbar_arrive_expect_tx(&bars.full[s], tx);
        tma_load_2d(st, &map_p, c * a.ncol + jb * PF_BK, (int)row0, &bars.full[s]);
        for (int i = 0; i < nbox; ++i)
          tma_load_2d_hint(st + PF_BM * 128 + i * 64 * 128, &map_k, n0 + i * 64, y, &bars.full[s], stream);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(UMMA_F16, UMMA_F16, PF_BM, nt, 1);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % PF_R_STAGES, use = kb / PF_R_STAGES;
        if (!mbar_wait_bounded(&bars.full[s], use & 1) || *bars.abort_flag) { *bars.abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * PF_R_STAGE);
        const uint32_t bk = st + PF_BM * 128;
#pragma unroll
        for (int ks = 0; ks < PF_BK / 16; ++ks)  // 16 slots per k-step: A +32 B along its row, B +16 rows (2 KB)
          tc_mma<0>(taddr, umma_desc_k_sw128(st + ks * 32), umma_desc_mn_sw128(bk + ks * 2048, 64 * 128), idesc,
                    kb > 0 || ks > 0);
        tc_commit(&bars.empty[s]);
      }
      tc_commit(bars.done);
    }
  } else {
    const int q4 = warp & 3;
    const int rr = q4 * 32 + lane;
    const int64_t t = row0 + rr;
    const bool row_ok = t0 + rr < a.rows_per_lib && t < a.n_rows;
    const bool ok = nkb > 0 && mbar_wait_bounded(bars.done, 0) && !*bars.abort_flag;
    tc_fence_after();
    const uint32_t tl = taddr + ((uint32_t)(q4 * 32) << 16);
    float* dst = a.r_out + t * a.d_s + n0;
    for (int c0 = 0; c0 < nt; c0 += 32) {
      float v[32];
      tc_ld32(tl + (uint32_t)c0, v);
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + c0 + i) =
              ok ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tc_dealloc(taddr, 256);
}

// The read as CTA pairs (2-CTA cluster, cta_group::2): CTAs 2p and 2p + 1 take token tiles 2p and 2p + 1 and the
// same 512 columns of d_s. Each loads its own 128 rows of P and, of each 256-column half, its 128 columns of the
// slots (the even CTA the first 128); the even CTA issues M = 256, N = 256 MMAs over both CTAs' shared memory into
// each CTA's 512 TMEM columns. Per SM and 64-slot k-block that is 48 KiB of operands for 128 x 512 x 64 MACs,
// half of what the single-CTA kernel moves for the same work, so the 4-stage ring covers twice the latency.
// Barriers as in a pair: both CTAs' copies count on the even CTA's full barrier, its commits arrive on both
// CTAs' empty and done barriers; TMEM is allocated and freed by warp 1 of both CTAs. d_s % 512 == 0.
constexpr int PF2R_BN = 512;                          // columns of d_s per pair
constexpr int PF2R_A = PF_BM * 128;                   // P: 128 rows x 64 slots
constexpr int PF2R_B = 4 * 64 * 128;                  // this CTA's 4 boxes of 64 columns x 64 slots
constexpr int PF2R_STAGE = PF2R_A + PF2R_B;
constexpr int PF2R_STAGES = 4;
constexpr size_t PF2R_SMEM = 1024 + (size_t)PF2R_STAGES * PF2R_STAGE + 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PF_THREADS, 1)
    prefill_read_pair_kernel(const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_k,
                             const PrefillArgs a) {
  extern __shared__ unsigned char pf_smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~uintptr_t(1023));
  const PfBars bars = pf_bars(smem + PF2R_STAGES * PF2R_STAGE, PF2R_STAGES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int64_t lib = blockIdx.z;
  const int n0 = blockIdx.y * PF2R_BN;
  const int64_t t0 = (int64_t)blockIdx.x * PF_BM;
  const int64_t row0 = lib * a.rows_per_lib + t0;
  const int nc = a.n_chunks_of ? min(a.n_chunks_of[lib], a.n_chunks) : a.n_chunks;
  const int kpc = a.ncol / PF_BK;  // k-blocks per chunk
  const int nkb = nc * kpc;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_p);
    prefetch_tensormap(&map_k);
  }
  if (warp == 1) {
    tc_alloc_cg2(bars.tmem_slot, 512);
    tc_relinquish_cg2();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < PF2R_STAGES; ++i) {
      mbar_init(&bars.full[i], 1);
      mbar_init(&bars.empty[i], 1);
    }
    mbar_init(bars.done, 1);
    *bars.abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the even CTA's barriers are initialised before the odd CTA's copies count on them
  tc_fence_after();
  const uint32_t taddr = *bars.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t stream = policy_evict_first();
      const uint32_t tx = 2u * (uint32_t)PF2R_STAGE;  // both CTAs' bytes land on the even CTA's barrier
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % PF2R_STAGES, use = kb / PF2R_STAGES;
        if (use > 0 && (!mbar_wait_bounded(&bars.empty[s], (use - 1) & 1) || *bars.abort_flag)) {
          *bars.abort_flag = 1;
          break;
        }
        const int c = kb / kpc, jb = kb - c * kpc;
        const int64_t page = a.page_of[lib * a.n_chunks + c];
        // P is 0 for a bad page (the scores kernel flagged it); its rows are read from past the pool (zeros)
        const int y = (page >= 0 && page < a.n_pages ? (int)(page * a.page_rows) : (int)(a.n_pages * a.page_rows)) +
                      jb * PF_BK;
        unsigned char* st = smem + s * PF2R_STAGE;
        const uint32_t fb = cluster_map(&bars.full[s], 0);
        if (rank == 0) mbar_arrive_expect_tx(&bars.full[s], tx);
        tma_load_2d_cg2(st, &map_p, c * a.ncol + jb * PF_BK, (int)row0, fb);
        for (int h = 0; h < 2; ++h)
          for (int i = 0; i < 2; ++i)
            tma_load_2d_cg2_hint(st + PF2R_A + (2 * h + i) * 64 * 128, &map_k, n0 + 256 * h + (int)rank * 128 + 64 * i,
                                 y, fb, stream);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = umma_idesc(UMMA_F16, UMMA_F16, 2 * PF_BM, 256, 1);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % PF2R_STAGES, use = kb / PF2R_STAGES;
        if (!mbar_wait_bounded(&bars.full[s], use & 1) || *bars.abort_flag) { *bars.abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * PF2R_STAGE);
#pragma unroll
        for (int ks = 0; ks < PF_BK / 16; ++ks) {  // 16 slots per k-step: A +32 B along its row, B +16 rows (2 KB)
          const uint64_t ad = umma_desc_k_sw128(st + ks * 32);
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tc_mma_cg2(taddr + 256u * h, ad, umma_desc_mn_sw128(st + PF2R_A + 2 * h * 64 * 128 + ks * 2048, 64 * 128),
                       idesc, kb > 0 || ks > 0);
        }
        tc_commit_cg2_mc(&bars.empty[s], 3);
      }
      tc_commit_cg2_mc(bars.done, 3);
    }
  } else {
    const int q4 = warp & 3;
    const int rr = q4 * 32 + lane;
    const int64_t t = row0 + rr;
    const bool row_ok = t0 + rr < a.rows_per_lib && t < a.n_rows;
    const bool ok = nkb > 0 && mbar_wait_bounded(bars.done, 0) && !*bars.abort_flag;
    tc_fence_after();
    const uint32_t tl = taddr + ((uint32_t)(q4 * 32) << 16);
    float* dst = a.r_out + t * a.d_s + n0;
    for (int c0 = 0; c0 < PF2R_BN; c0 += 32) {
      float v[32];
      tc_ld32(tl + (uint32_t)c0, v);
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + c0 + i) =
              ok ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA frees TMEM or leaves while the pair's MMAs or the other epilogue may run
  tc_fence_after();
  if (warp == 1) tc_dealloc_cg2(taddr, 512);
}

// q (f32) -> f16 for the scores product.
__global__ void __launch_bounds__(256) to_f16_kernel(const float* __restrict__ x, int64_t n, __half* __restrict__ y) {
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n; i += (int64_t)gridDim.x * blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    float r0, r1, r2, r3;
    uint2 o;
    o.x = pack2<__half>(v.x, v.y, r0, r1);
    o.y = pack2<__half>(v.z, v.w, r2, r3);
    *reinterpret_cast<uint2*>(y + i) = o;
  }
}

}  // namespace xencb

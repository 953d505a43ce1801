// Exchange of the chunk-sharded read's partial blocks over NVLink peer memory, in place of an
// all-gather: every rank pushes its block straight into every rank's exchange buffer with plain peer stores, and
// the merge waits for the blocks' flags before it combines them (the shard merge of read_multi.cuh).
//
// Exchange buffer of one rank (allocated by xencb_exch_alloc, mapped into the other ranks by CUDA IPC):
//   [0, EX_FLAG_BYTES)   flags: uint32 per (source rank, slice), the epoch of the last slice delivered here
//   then                 blocks: [2 parities][G ranks][per floats], the block of epoch e in parity e & 1
// A block travels as EX_SLICES slices, one CTA each, so a push keeps G * EX_SLICES SMs storing over NVLink.
// Local state of a rank (3 uint32, zero at start): [0] the epoch of the last push, [1] the epoch the next merge
// reads, [2] the push kernel's CTA counter.
//
// Epochs order the steps without a reset: push n writes epoch n into parity n & 1 of every rank and raises the
// flags to n; merge n waits for every flag >= n. A rank can be at most one step ahead of another rank's merge
// (its push n + 1 follows its own merge n, which waited for that rank's push n, which followed that rank's merge
// n - 1), so the two parities never hold a block that is still being read. Every wait is bounded: a flag that
// does not arrive within XENCB_WAIT_CYCLES sets XENCB_DEV_TIMEOUT and the merge goes on with what is there.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace xencb {

constexpr int EX_SLICES = 8;
constexpr int EX_MAX_RANKS = 64;
constexpr int EX_FLAG_BYTES = EX_MAX_RANKS * EX_SLICES * 4;
constexpr int EX_PUSH_THREADS = 256;

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid (G, EX_SLICES): CTA (d, s) copies slice s of this rank's block (per floats) into parity e & 1, slot
// `rank`, of rank d's buffer, then raises rank d's flag for (rank, s) to e. The last CTA to finish advances the
// local epochs.
__global__ void __launch_bounds__(EX_PUSH_THREADS) shard_push_kernel(const float* __restrict__ block, int64_t per,
                                                                     const uint64_t* __restrict__ peers, int G,
                                                                     int rank, uint32_t* __restrict__ state) {
  const int dst = blockIdx.x, sl = blockIdx.y;
  const uint32_t e = state[0] + 1u;  // every CTA reads it before the last one moves it
  char* base = reinterpret_cast<char*>(peers[dst]);
  float* slot = reinterpret_cast<float*>(base + EX_FLAG_BYTES) + ((int64_t)(e & 1u) * G + rank) * per;
  if ((per & 3) == 0 && (reinterpret_cast<uintptr_t>(block) & 15) == 0) {
    const int64_t n4 = per / 4, c4 = (n4 + EX_SLICES - 1) / EX_SLICES;
    const int64_t i0 = sl * c4, i1 = min(n4, i0 + c4);
    const float4* s4 = reinterpret_cast<const float4*>(block);
    float4* d4 = reinterpret_cast<float4*>(slot);
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) d4[i] = __ldg(s4 + i);
  } else {
    const int64_t c1 = (per + EX_SLICES - 1) / EX_SLICES;
    const int64_t i0 = sl * c1, i1 = min(per, i0 + c1);
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) slot[i] = __ldg(block + i);
  }
  __threadfence_system();  // this thread's stores reach the peer before the flag below
  __syncthreads();
  if (threadIdx.x == 0) {
    st_release_sys_u32(reinterpret_cast<uint32_t*>(base) + rank * EX_SLICES + sl, e);
    __threadfence();
    if (atomicAdd(&state[2], 1u) == (uint32_t)(G * EX_SLICES) - 1u) {
      state[2] = 0u;
      state[1] = e;
      state[0] = e;
    }
  }
}

// The shard merge over the G blocks of epoch state[1] in this rank's exchange buffer, after its flags arrived:
// r = sum_g e^(M_g - M) A_g / sum_g e^(M_g - M) Z_g (the blocks as shard_merge_kernel reads them). Grid (rows,
// column blocks); each CTA waits for the flags, the blocks are read through L2 (written by peers).
__global__ void __launch_bounds__(256) shard_merge_wait_kernel(const char* __restrict__ exch, int G, int64_t n_rows,
                                                               int d_s, const uint32_t* __restrict__ state,
                                                               float* __restrict__ r_out) {
  const int64_t row = blockIdx.x;
  const int64_t per = n_rows * 4 + n_rows * (int64_t)d_s;
  const uint32_t e = state[1];
  const float* parts = reinterpret_cast<const float*>(exch + EX_FLAG_BYTES) + (int64_t)(e & 1u) * G * per;
  // thread t waits for flags t, t + blockDim.x, ... (the G * EX_SLICES slices), all in parallel
  {
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(exch);
    const long long t0 = clock64();
    for (int f = threadIdx.x; f < G * EX_SLICES; f += blockDim.x) {
      for (uint32_t it = 0;; ++it) {
        if ((int32_t)(ld_acquire_sys_u32(flags + f) - e) >= 0) break;
        if ((it & 63u) == 63u && clock64() - t0 > XENCB_WAIT_CYCLES) {
          flag_error(XENCB_DEV_TIMEOUT);
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  float Mx = -CUDART_INF_F;
  for (int g = 0; g < G; ++g) Mx = fmaxf(Mx, __ldcg(parts + g * per + row * 4));
  float den = 0.f;
  for (int g = 0; g < G; ++g) {
    const float* h = parts + g * per + row * 4;
    const float z = __ldcg(h + 1);
    if (z > 0.f) den += expf(__ldcg(h) - Mx) * z;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int d = blockIdx.y * blockDim.x + threadIdx.x; d < d_s; d += gridDim.y * blockDim.x) {
    float num = 0.f;
    for (int g = 0; g < G; ++g) {
      const float* h = parts + g * per + row * 4;
      if (__ldcg(h + 1) > 0.f) num += expf(__ldcg(h) - Mx) * __ldcg(parts + g * per + n_rows * 4 + row * d_s + d);
    }
    r_out[row * d_s + d] = num * inv;
  }
}

}  // namespace xencb

// Shared device helpers for the xencb kernels (sm_100a only).
//
// * dtype codes and vector loads for hidden states / slots,
// * mbarrier + cp.async.bulk (1-D TMA, no multicast) primitives in inline PTX,
// * bounded waits: every spin on an mbarrier gives up after XENCB_WAIT_CYCLES SM cycles (1.5 s at 2 GHz), records
//   XENCB_DEV_TIMEOUT in the per-device status word and lets the kernel return.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/xencb.h"


namespace xencb {

// Per-device status word (bit flags, see xencb.h XENCB_DEV_*). Read and cleared by xencb_device_status().
// The library is one translation unit (xencb.cu includes every kernel header), so this is its definition.
__device__ unsigned int g_dev_status = 0;

__device__ __forceinline__ void flag_error(unsigned int bits) { atomicOr(&g_dev_status, bits); }

// Programmatic dependent launch (the kernels the host launches with programmatic stream serialisation: the read
// merge, the row split, the 3xF16 GEMM, the projection row kernels and the fused decode router). pdl_wait()
// returns once the grid before this one in the stream has completed and its writes are visible (a no-op for a
// plain launch). Before it such a kernel only reads, and only data that no kernel still running can be writing:
// the GEMM's weight tiles and the router's summary keys (Library data), and the row kernels' hidden-state rows
// (they start after the GEMM has passed its own wait, so the kernel that wrote h has completed). Nothing is written
// before the wait. pdl_trigger() lets the next grid be scheduled; the row split and the row kernels issue it first
// thing (their successors' early work is such a read), the others after their wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------ dtypes
template <typename T> struct DT;
template <> struct DT<float> { static constexpr int code = XENCB_F32; };
template <> struct DT<__half> { static constexpr int code = XENCB_F16; };
template <> struct DT<__nv_bfloat16> { static constexpr int code = XENCB_BF16; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Unpack one 16-byte vector into floats: 4 (f32) or 8 (f16 / bf16) elements.
template <typename T> struct Vec16 { static constexpr int n = 16 / sizeof(T); };

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float* out);

template <>
__device__ __forceinline__ void unpack16<float>(const uint4& v, float* out) {
  out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
  out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}

template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& v, float* out) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    out[2 * i] = f.x; out[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& v, float* out) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    out[2 * i] = f.x; out[2 * i + 1] = f.y;
  }
}

// ------------------------------------------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` must hold 32 floats. Result broadcast to all threads.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// ------------------------------------------------------------------------------------------------ mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy that bypasses registers (cp.async, completion per thread by wait_all).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n\tcp.async.commit_group;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with parity `parity` of `bar` completed. Returns false (and flags the device status)
// if it did not happen within XENCB_WAIT_CYCLES; the caller must then stop using the pipeline.
// The retries pass a suspend-time hint, so a waiting thread sleeps in the barrier instead of spinning, and the
// clock is read only every 16th retry: a warp waiting here takes almost no issue slots from working warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

// The limit is counted on the SM's cycle counter (cheap to read, unlike the global timer, whose reads cost more
// than a whole pipeline hand-off): XENCB_WAIT_CYCLES is 1.5 s at 2 GHz, longer in time at lower clocks.
#ifndef XENCB_WAIT_CYCLES
#define XENCB_WAIT_CYCLES 3000000000ll
#endif

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((it & 15u) == 0u && clock64() - t0 > XENCB_WAIT_CYCLES) {
      flag_error(XENCB_DEV_TIMEOUT);
      return false;
    }
  }
}

// The same bounded wait without the suspend hint: for short waits on a hot path (a phase that other warps are
// about to complete), where a suspended thread's wake-up would cost more than the few retries it saves.
__device__ __forceinline__ bool mbar_wait_spin_limit(uint64_t* bar, uint32_t parity, long long limit_cycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u && clock64() - t0 > limit_cycles) {
      flag_error(XENCB_DEV_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity) {
  return mbar_wait_spin_limit(bar, parity, XENCB_WAIT_CYCLES);
}

// 1-D bulk copy global -> this CTA's shared memory, completion signalled on `bar` as transaction bytes.
// `bytes` and both addresses must be multiples of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Ask L2 to fetch [gmem_src, gmem_src + bytes) from HBM (no shared memory, no completion to wait for): a later
// copy of the same bytes finds them in L2. `bytes` and the address must be multiples of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* gmem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------------ mma.sync
// ldmatrix: four 8x8 b16 matrices; lane l supplies the row address of matrix l/8, row l%8.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Transpose an 8x8 b16 matrix held in mma fragment layout across the warp.
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// D (16x8 f32) += A (16x16) * B (16x8); A/B f16 or bf16.
template <typename T>
__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__half>(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Pack two floats into one b32 of T (low half = first) and return the rounded values.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y, float& rx, float& ry) {
  const T hx = from_f32<T>(x), hy = from_f32<T>(y);
  rx = to_f32(hx);
  ry = to_f32(hy);
  uint16_t ux, uy;
  memcpy(&ux, &hx, 2);
  memcpy(&uy, &hy, 2);
  return (uint32_t)ux | ((uint32_t)uy << 16);
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace xencb

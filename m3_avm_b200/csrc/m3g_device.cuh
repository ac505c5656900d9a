// m3g_device.cuh -- device-side helpers shared by the m3gemv kernels (sm_100a).
//
// - exact f16 -> f32 widening of the GGUF block scales;
// - byte -> float conversion without I2F: a byte placed in the low mantissa
//   of 2^23 (0x4B0000bb) is exactly 2^23 + b, so one PRMT plus one FADD of a
//   constant turns a packed quant into its exact float value (bias included);
// - 1-D TMA bulk copies global -> shared completed on an mbarrier, and a
//   bounded mbarrier wait that reports instead of hanging.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace m3g {

__device__ __forceinline__ float f16_to_f32(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// Byte k (0..3) of w as the float 2^23 + byte.  Subtracting (2^23 + bias)
// afterwards yields byte - bias exactly for any bias in [0, 255].
template <int K>
__device__ __forceinline__ float byte_2p23(uint32_t w) {
  return __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7540u | K)));
}
__device__ __forceinline__ float byte_2p23_rt(uint32_t w, int k) {
  return __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7540u | static_cast<unsigned>(k))));
}
constexpr float k2p23 = 8388608.0f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// N 32-bit words starting at an arbitrary byte address p in shared memory.
// Reads the aligned words covering [p, p + 4N + 3]; callers keep 16 bytes of
// slack after every buffer they read this way.
template <int N>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t (&out)[N]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  uint32_t w[N + 1];
#pragma unroll
  for (int i = 0; i <= N; ++i) w[i] = base[i];
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses (made
// visible to it by a CTA barrier) before its later async-proxy (TMA) writes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar`.  dst/src 16-byte aligned, bytes % 16 == 0.
// No multicast: the source is always this GPU's own memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar` to complete, giving up after ~timeout_ns
// of wall time or 2^26 polls, whichever comes first, or as soon as another
// thread of the CTA has raised *abort (checked every 256 polls).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t timeout_ns,
                                                  const volatile int* abort = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1; it < (1u << 26); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > timeout_ns) return false;
    }
  }
  return false;
}

// System-scope acquire load of a counter that other GPUs increment.
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until *cnt has reached target (wrap-safe), giving up after ~timeout_ns
// of wall time or 2^24 polls.  Returns false when it gave up.
__device__ __forceinline__ bool wait_count_bounded(const unsigned int* cnt, unsigned int target,
                                                   uint64_t timeout_ns) {
  if (static_cast<int>(ld_acquire_sys(cnt) - target) >= 0) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1; it < (1u << 24); ++it) {
    __nanosleep(32);
    if (static_cast<int>(ld_acquire_sys(cnt) - target) >= 0) return true;
    if ((it & 63u) == 0u && global_ns() - t0 > timeout_ns) return false;
  }
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Named barrier over the first `count` threads' warps that execute it (id 1..15).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Programmatic dependent launch: block until the grids this launch depends on
// have completed and flushed memory (no-op for an ordinary launch), and allow
// the next dependent grid to begin its pre-wait prologue.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// x -> three int8 slices of super-block sb and its group sums; lane holds
// elements 8*lane .. 8*lane+7 in v.
__device__ __forceinline__ void quantize_sb(const float (&v)[8], int sb, int lane, uint8_t* xsl, float* sum32,
                                            float* sum16, float* sxs) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const float inv = amax > 0.f ? 127.0f / amax : 0.f;
  uint32_t s0[2] = {0u, 0u}, s1[2] = {0u, 0u}, s2[2] = {0u, 0u};
  float part = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    part += v[i];
    const float q = v[i] * inv;
    const float q0 = rintf(q);
    const float u1 = (q - q0) * 254.0f;
    const float q1 = rintf(u1);
    const float q2 = rintf((u1 - q1) * 254.0f);
    const int sh = 8 * (i & 3);
    s0[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q0)) & 0xFFu) << sh;
    s1[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q1)) & 0xFFu) << sh;
    s2[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q2)) & 0xFFu) << sh;
  }
  // lane covers elements 8*lane .. +8: sub-block j = lane / 4, offset 8 * (lane % 4)
  uint8_t* dst = xsl + (static_cast<size_t>(sb) * 8 + (lane >> 2)) * 96 + 8 * (lane & 3);
  *reinterpret_cast<uint2*>(dst) = make_uint2(s0[0], s0[1]);
  *reinterpret_cast<uint2*>(dst + 32) = make_uint2(s1[0], s1[1]);
  *reinterpret_cast<uint2*>(dst + 64) = make_uint2(s2[0], s2[1]);
  const float p16 = part + __shfl_xor_sync(0xFFFFFFFFu, part, 1);
  if ((lane & 1) == 0) sum16[sb * 16 + (lane >> 1)] = p16;
  const float p32 = p16 + __shfl_xor_sync(0xFFFFFFFFu, p16, 2);
  if ((lane & 3) == 0) sum32[sb * 8 + (lane >> 2)] = p32;
  if (lane == 0) sxs[sb] = amax > 0.f ? amax / 127.0f : 0.f;
}


}  // namespace m3g

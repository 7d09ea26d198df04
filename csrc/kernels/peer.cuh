// Device helpers for kernels that load and store other GPUs' memory over NVLink:
// bounded waits on flags written by peers (global timer budget), system-scope
// release/acquire, uncached loads of peer-written data, and "flag-in-data" words and
// lines (32-bit payloads each paired with the call's epoch in one 8-byte half, so a reader
// never pairs the payload of one call with the flag of another).
#pragma once
#include "sm100_common.cuh"

namespace zs {
namespace peer {

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t limit_ns(unsigned int timeout_ms) {
  return (uint64_t)(timeout_ms ? timeout_ms : 5000u) * 1000000ull;
}


__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Uncached 16-byte load (peer data written by another GPU since our last read).
__device__ __forceinline__ uint4 ld_cv_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cv.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

// Spin until `*p - value >= 0` (wrap-safe) or `budget_ns` passes; acquire at system scope.
__device__ __forceinline__ bool wait_flag_sys(const uint32_t* p, uint32_t value, uint64_t budget_ns,
                                              const int* abort_word) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if ((int)(ld_acquire_sys(p) - value) >= 0) return true;
    if (abort_word && *reinterpret_cast<const volatile int*>(abort_word)) return false;
    if (i > 32) {
      __nanosleep(64);
      if ((i & 255) == 0 && globaltimer_ns() - t0 > budget_ns) return false;
    }
  }
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 v = __bfloat1622float2(h[j]);
    f[2 * j] = v.x;
    f[2 * j + 1] = v.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint32_t p[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    p[j] = *reinterpret_cast<uint32_t*>(&b);
  }
  return make_uint4(p[0], p[1], p[2], p[3]);
}

// Flag-in-data word: 32 bits of payload (two bf16) + the call's epoch, stored with one
// 8-byte store so a reader never sees the payload of one call with the flag of another.
__device__ __forceinline__ void st_ll(uint2* p, uint32_t data, uint32_t epoch) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(epoch) : "memory");
}
__device__ __forceinline__ uint2 ld_ll(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// Waits for the word at p to carry `epoch`; returns its payload (0 and an error on timeout).
__device__ __forceinline__ uint32_t wait_ll(const uint2* p, uint32_t epoch, uint64_t budget_ns, int* err,
                                            volatile int* give_up) {
  uint2 v = ld_ll(p);
  if (v.y == epoch) return v.x;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    v = ld_ll(p);
    if (v.y == epoch) return v.x;
    if (*give_up) return 0u;
    if ((i & 63) == 63) {
      if (globaltimer_ns() - t0 > budget_ns) {
        report_error(err, kErrPeerTimeout);
        *give_up = 1;
        return 0u;
      }
      __nanosleep(32);
    }
  }
}

// 16-byte LL line {d0, epoch, d1, epoch}: two 32-bit payload words, each paired with the
// call's epoch in one 8-byte half, stored with one vector store.  A reader accepts the line
// only when both halves carry the current epoch.
__device__ __forceinline__ void st_ll16(void* p, uint32_t d0, uint32_t d1, uint32_t e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(d0), "r"(e), "r"(d1), "r"(e)
               : "memory");
}
__device__ __forceinline__ uint4 ld_ll16(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool ll_ok(const uint4& v, uint32_t e) { return v.y == e && v.w == e; }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}

}  // namespace peer
}  // namespace zs

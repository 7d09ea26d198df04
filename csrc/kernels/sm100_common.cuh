// Blackwell (sm_100a) device helpers shared by every zstep_b200 kernel.
//
// Everything here is a thin inline-PTX wrapper around the tcgen05 / TMA / mbarrier
// instruction families, plus the bounded-wait discipline every kernel follows:
// no spin loop in this library is unbounded.  A wait that runs out of iterations
// records an error code in a device-global error word (read by the host after the
// step) and returns false, and the caller unwinds (drains its own copies, frees TMEM,
// returns) instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#define ZS_DEVICE __device__ __forceinline__

namespace zs {

// ---------------------------------------------------------------------------------
// Error reporting.  Codes are small positive integers; the first error wins.
// ---------------------------------------------------------------------------------
enum ErrorCode : int {
  kErrNone = 0,
  kErrMbarTimeout = 1,     // an mbarrier wait ran out of iterations
  kErrPeerTimeout = 2,     // a cross-GPU flag wait ran out of iterations
  kErrBadShape = 3,        // a kernel saw an argument outside its contract
  kErrDrainTimeout = 4,    // teardown could not drain in-flight copies in time
  kErrAbort = 5,           // host-set abort word observed
};

ZS_DEVICE void report_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// Iteration cap for mbarrier waits.  Each failed try_wait is followed by a short
// nanosleep, so 1<<22 iterations is on the order of a second: far above any legal
// wait inside a kernel, far below a watchdog.
constexpr uint32_t kMbarSpinLimit = 1u << 22;

ZS_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

ZS_DEVICE bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

ZS_DEVICE int warp_id() { return __shfl_sync(0xffffffff, threadIdx.x / 32, 0); }
ZS_DEVICE int lane_id() { return threadIdx.x & 31; }

// ---------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------
ZS_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

ZS_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

ZS_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

ZS_DEVICE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

ZS_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records kErrMbarTimeout) if the phase never
// completes within kMbarSpinLimit tries.
ZS_DEVICE bool mbar_wait(uint64_t* bar, uint32_t phase, int* err) {
  for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
    if (i > 64) __nanosleep(128);
  }
  report_error(err, kErrMbarTimeout);
  return false;
}

// ---------------------------------------------------------------------------------
// TMA (non-multicast only: this library never issues a cluster-multicast load).
// ---------------------------------------------------------------------------------
ZS_DEVICE void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(desc) : "memory");
}

// 2-D tiled load: coordinates are (x = innermost, y).  The caller guarantees that
// x * element_size is a multiple of 16 bytes.
ZS_DEVICE void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

ZS_DEVICE void tma_load_3d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Untiled bulk copy global -> shared; both addresses 16-byte aligned, bytes % 16 == 0.
ZS_DEVICE void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

ZS_DEVICE void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, copies and loads.
// ---------------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32).  Must be executed by one
// full warp; the base address is written to *dst_smem.
ZS_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

ZS_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

ZS_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

ZS_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
ZS_DEVICE void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive on an mbarrier once every tcgen05 op previously issued by this thread completes.
ZS_DEVICE void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), bf16/f16 inputs, f32 accumulate.
ZS_DEVICE void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Block-scaled MXFP8 MMA: A/B e4m3 in smem, per-32-K e8m0 scales in TMEM.
ZS_DEVICE void mma_mxf8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                        uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Copy a 32-row x 16-byte block from shared memory into 4 TMEM columns, replicated
// into all four 32-lane subpartitions (the scale-factor staging copy).
ZS_DEVICE void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t src_desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc)
               : "memory");
}

// Each thread of a warp reads 16 consecutive 32-bit columns of its own TMEM lane.
ZS_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

ZS_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

ZS_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Each thread of a warp writes 16 consecutive 32-bit columns of its own TMEM lane.
ZS_DEVICE void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
ZS_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for tcgen05 (sm_100 layout: version field = 1).
//   layout: 0 = no swizzle (canonical 8x16B core matrices), 2 = 128-byte swizzle.
ZS_DEVICE uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                  uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 0x7) << 61;
  return d;
}

// Instruction descriptor for kind::mxf8f6f4.block_scale with e4m3 A/B, K-major
// operands, e8m0 scales, f32 accumulator.  sf ids select the byte of the 32-bit
// TMEM scale column used by this MMA.
ZS_DEVICE uint32_t make_idesc_mxf8(uint32_t M, uint32_t N, uint32_t a_sf_id, uint32_t b_sf_id) {
  uint32_t d = 0;
  d |= (b_sf_id & 3u) << 4;
  // a_format (bits 7-9) = 0 (E4M3), b_format (bits 10-12) = 0 (E4M3), K-major both.
  d |= ((N >> 3) & 0x3Fu) << 17;
  d |= 1u << 23;  // scale factor type = UE8M0
  d |= ((M >> 4) & 0x1Fu) << 24;
  d |= (a_sf_id & 3u) << 29;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, f32 accumulator.
//   a_mn_major / b_mn_major: 0 = K-major, 1 = MN-major.
ZS_DEVICE uint32_t make_idesc_bf16(uint32_t M, uint32_t N, uint32_t a_mn_major,
                                   uint32_t b_mn_major) {
  uint32_t d = 0;
  d |= 1u << 4;   // D format f32
  d |= 1u << 7;   // A bf16
  d |= 1u << 10;  // B bf16
  d |= (a_mn_major & 1u) << 15;
  d |= (b_mn_major & 1u) << 16;
  d |= ((N >> 3) & 0x3Fu) << 17;
  d |= ((M >> 4) & 0x1Fu) << 24;
  return d;
}

// ---------------------------------------------------------------------------------
// Small numeric helpers.
// ---------------------------------------------------------------------------------
ZS_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

ZS_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

ZS_DEVICE float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
ZS_DEVICE float siluf_(float x) { return x / (1.0f + __expf(-x)); }

// E8M0 block scale for an MXFP8 (e4m3) block with absolute maximum `amax`.
// The scale is the power of two 2^e with e = ceil(log2(amax / 448)), so that every
// scaled element fits the e4m3 range (max finite 448); e is clamped to [-127, 127]
// and encoded with bias 127.  Computed exactly from the float's exponent bits.
ZS_DEVICE uint8_t mx_scale_e8m0(float amax) {
  if (!(amax > 0.0f)) return 0;  // zero block: any scale works, use the smallest
  float r = amax * (1.0f / 448.0f);
  uint32_t bits = __float_as_uint(r);
  int e = static_cast<int>((bits >> 23) & 0xFF) - 127;
  if ((bits & 0x7FFFFF) != 0) e += 1;  // ceil for non powers of two
  if (e < -127) e = -127;
  if (e > 127) e = 127;
  return static_cast<uint8_t>(e + 127);
}

// 1 / 2^(code-127) as a float (exact power of two).
ZS_DEVICE float mx_inv_scale(uint8_t code) {
  int e = 127 - (static_cast<int>(code) - 127);  // biased exponent of 2^-(code-127)
  if (e <= 0) return 0.0f;
  if (e >= 255) e = 254;
  return __uint_as_float(static_cast<uint32_t>(e) << 23);
}

ZS_DEVICE float mx_scale_value(uint8_t code) {
  int e = static_cast<int>(code);
  if (e == 0) return __uint_as_float(0x00400000u);  // 2^-127 (denormal)
  return __uint_as_float(static_cast<uint32_t>(e) << 23);
}

ZS_DEVICE uint8_t f32_to_e4m3(float v) {
  __nv_fp8_e4m3 q(v);  // saturating round-to-nearest-even conversion
  return *reinterpret_cast<uint8_t*>(&q);
}

// Argmax key: high word = logit bits mapped to an unsigned order, low word = ~id,
// so an unsigned max picks the largest logit and, among equal logits, the smallest id.
// Gumbel(0, 1) noise for sampling by perturbed argmax: the same (seed, position, token
// id) gives the same noise on every rank, so a vocab-sharded lm_head samples one token
// consistently.  Uniform from one SplitMix64 step (24-bit mantissa, open interval).
ZS_DEVICE float gumbel_noise(unsigned long long seed, int pos, int id) {
  unsigned long long z = seed ^ ((unsigned long long)(unsigned)pos * 0x9E3779B97F4A7C15ull) ^
                         ((unsigned long long)(unsigned)id * 0xD1B54A32D192ED03ull);
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  const float u = ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

ZS_DEVICE unsigned long long pack_argmax(float v, int id) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | static_cast<uint32_t>(~id);
}

ZS_DEVICE float unpack_argmax_value(unsigned long long key) {
  uint32_t b = static_cast<uint32_t>(key >> 32);
  b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
  return __uint_as_float(b);
}

ZS_DEVICE int unpack_argmax_id(unsigned long long key) {
  return static_cast<int>(~static_cast<uint32_t>(key & 0xFFFFFFFFull));
}

// Byte offset of (row, k) inside the 128-row x 4-block scale atom (512 bytes) used by
// the MXFP8 GEMM: rows r = r0 + 32*r1 live in 16-byte line r0, byte r1*4 + kblk.
ZS_DEVICE int sf_atom_offset(int row_in_atom, int kblk_in_atom) {
  return (row_in_atom & 31) * 16 + (row_in_atom >> 5) * 4 + kblk_in_atom;
}

// ---------------------------------------------------------------------------------
// Programmatic dependent launch.  Kernels started by zs_launch may begin while the
// previous kernel of the stream is still running (its CTAs free SMs one by one), so the
// launch, the CTA ramp and a kernel's local set-up overlap the predecessor's tail.  Every
// such kernel calls pdl_wait() before it touches global memory that an earlier kernel
// writes or reads, and pdl_trigger() to let its own successor launch early.  Both are
// no-ops for a kernel launched without the attribute.
// ---------------------------------------------------------------------------------
ZS_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
ZS_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace zs

// Host switch (zs_set_pdl) and the launcher used by every kernel that waits with pdl_wait.
extern "C" int zs_pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t zs_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = zs_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

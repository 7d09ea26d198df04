// Tensor-parallel collectives fused with their consumers, over NVLink peer memory.
//
// Symmetric memory: every rank allocates the same buffers with cudaMalloc and maps its
// peers' copies through CUDA IPC (cudaIpcOpenMemHandle), so a kernel on rank r stores
// straight into rank q's buffer over NVLink / NVSwitch.  Every protocol here is
// push-based: a kernel only ever stores to peers and loads its own memory, so each
// NVLink crossing is one posted write and no load waits on a remote round trip.
//
// LL lines.  Decode-sized messages move as 16-byte "LL lines" {d0, epoch, d1, epoch}: two
// 32-bit payload words (four bf16, or two f32), each paired with the call's epoch in one
// 8-byte half.  A reader accepts a line only when both halves carry the current epoch,
// so data and flag arrive in the same store and no separate barrier round trip is paid.
// Readers issue the loads of every source before checking any (up to 8 in flight per
// thread), then re-poll only the stale ones: a wait costs one memory latency, not one per
// source.  Epochs are per-protocol device counters advanced by the last CTA of each call,
// so every call (eager or CUDA-graph replay) carries fresh flag values.
//
// fused_allreduce_norm, three protocols (host chooses by row count):
//   one-shot : every rank pushes its local rows to every rank (parity-double-buffered);
//              each rank sums residual + the W contributions in rank order.  One hop.
//   two-shot : reduce-scatter to the row's owner + all-gather of the owner's bf16 result,
//              both as LL lines.  Two hops, 2(W-1)/W of the bytes of the one-shot.
//   plain    : the two-shot data flow with plain bf16 rows and per-(source, CTA) flags
//              released after a system-scope fence, for prefill-sized reductions where
//              the LL format's doubled bytes would dominate.
//   nvls     : NVLink SHARP: the buffers are bound to an NVSwitch multicast object, the
//              switch sums the ranks' copies (multimem.ld_reduce) and broadcasts each
//              result (multimem.st); each rank reduces 1/world of the columns.
// All three then apply residual add, RMSNorm and MXFP8 quantization in the same kernel.
// Every rank computes every row's sum in the same order, so all ranks hold identical
// bf16 residual streams.
//
// allreduce_argmax: the lm_head's per-tile keys -> per-row key -> global ids -> one LL
// line per (row, rank) pushed to every rank -> max over ranks, in one kernel.
//
// allreduce_sum_f32: one-shot LL fp32 sum (the mHC model's sublayer outputs).
//
// Launch: all kernels use programmatic dependent launch (set-up overlaps the producer's
// tail; each waits before its first read of predecessor output).  A two-shot CTA c only
// waits for CTA c of other ranks (same row -> CTA map everywhere) and never for another
// CTA of its own rank, and FAR_CTAS CTAs of 256 threads with a few KB of shared memory fit
// beside any kernel of this library, so they are all resident without a cooperative launch.
//
// Reference parity: replaces worker/zstep_worker/kernels_sm120/csrc/shm_allreduce_kernels.cu
// (shm_v5 all-reduce :472, fused AR + add + RMSNorm :1376, spin-wait with abort :31-83)
// and the TP=8 argmax exchange (csrc/qwen35_ops_kernels.cu:202).
#include "peer.cuh"
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace coll {

constexpr int THREADS = 256;
constexpr int MAX_LPT = 4;  // LL lines (4 columns each) per thread per row: hidden <= 4096

using namespace peer;


// Loads the n (<= N) lines p[0], p[stride], ... and waits until every one carries epoch e.
// All loads are issued before any is checked; stale lines are re-polled until the time
// budget runs out (then kErrPeerTimeout, and the CTA-wide give_up word stops the others).
template <int N>
__device__ __forceinline__ bool wait_lines(const uint4* p, size_t stride, int n, uint32_t e, uint4 (&v)[N],
                                           uint64_t budget, int* err, volatile int* give_up) {
  uint32_t pend = 0;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n) v[i] = ld_ll16(p + i * stride);
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n && !ll_ok(v[i], e)) pend |= 1u << i;
  if (pend == 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if ((pend >> i) & 1u) {
        v[i] = ld_ll16(p + i * stride);
        if (ll_ok(v[i], e)) pend &= ~(1u << i);
      }
    if (pend == 0) return true;
    if (*give_up) return false;
    if ((it & 15) == 15) {
      if (globaltimer_ns() - t0 > budget) {
        report_error(err, kErrPeerTimeout);
        *give_up = 1;
        return false;
      }
      __nanosleep(32);
    }
  }
}

__device__ __forceinline__ float4 bf16x4_to_f4(uint32_t lo, uint32_t hi) {
  const float2 a = unpack_bf16x2(lo), b = unpack_bf16x2(hi);
  return make_float4(a.x, a.y, b.x, b.y);
}

// This rank's contribution to columns [4l, 4l + 4) of `row`: its terms summed in term order
// (fp32), as the caller will round it (bf16 on the wire).
__device__ __forceinline__ float4 local_line(const FusedArArgs& a, int row, int l) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  const int c = 4 * l;
  for (int t = 0; t < a.n_terms; ++t) {
    long long off = row * a.row_stride + t * a.term_stride + c;
    float sc = 1.f;
    if (a.term_index != nullptr) {  // gathered term; negative = not produced on this rank
      const int src = __ldg(a.term_index + row * a.n_terms + t);
      if (src < 0) continue;
      off = (long long)src * a.row_stride + c;
    }
    if (a.term_scale != nullptr) sc = __ldg(a.term_scale + row * a.n_terms + t);
    float4 v;
    if (a.delta_f32) {
      v = *reinterpret_cast<const float4*>(static_cast<const float*>(a.delta) + off);
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.delta) + off);
      v = bf16x4_to_f4(u.x, u.y);
    }
    s.x += sc * v.x;
    s.y += sc * v.y;
    s.z += sc * v.z;
    s.w += sc * v.w;
  }
  return s;
}

// Finishing step shared by every protocol, for one row whose reduced bf16 values this
// thread holds as lines l = tid + i * THREADS (i < lpt): write the residual, RMSNorm over
// the row (block reduction), then the bf16 and/or MXFP8 outputs.  An MXFP8 block of 32
// columns is 8 consecutive lines = 8 consecutive threads.
__device__ __forceinline__ void finish_row(const FusedArArgs& a, int row, int lpt, const uint2 (&res)[MAX_LPT],
                                           float* red) {
  const int H = a.hidden, tid = threadIdx.x;
  __nv_bfloat16* res_out = static_cast<__nv_bfloat16*>(a.residual) + (size_t)row * H;
  float x[MAX_LPT][4];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAX_LPT; ++i) {
    if (i >= lpt) break;
    const int c = 4 * (tid + i * THREADS);
    *reinterpret_cast<uint2*>(res_out + c) = res[i];
    const float4 f = bf16x4_to_f4(res[i].x, res[i].y);
    x[i][0] = f.x;
    x[i][1] = f.y;
    x[i][2] = f.z;
    x[i][3] = f.w;
    ss += f.x * f.x + f.y * f.y + f.z * f.z + f.w * f.w;
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) tot += red[i];
  __syncthreads();  // red is reused by the next row
  const float rstd = rsqrtf(tot / H + a.eps);
  const __nv_bfloat16* wgt = static_cast<const __nv_bfloat16*>(a.weight);
#pragma unroll
  for (int i = 0; i < MAX_LPT; ++i) {
    if (i >= lpt) break;
    const int c = 4 * (tid + i * THREADS);
    const uint2 wu = *reinterpret_cast<const uint2*>(wgt + c);
    const float4 w4 = bf16x4_to_f4(wu.x, wu.y);
    float y[4] = {x[i][0] * rstd * (w4.x + a.w_offset), x[i][1] * rstd * (w4.y + a.w_offset),
                  x[i][2] * rstd * (w4.z + a.w_offset), x[i][3] * rstd * (w4.w + a.w_offset)};
    if (a.normed)
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.normed) + (size_t)row * H + c) =
          make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
    if (a.q) {
      float amax = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 4));
      const uint8_t code = mx_scale_e8m0(amax);
      const float inv = mx_inv_scale(code);
      uint32_t pk = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) pk |= uint32_t(f32_to_e4m3(y[j] * inv)) << (8 * j);
      *reinterpret_cast<uint32_t*>(a.q + (size_t)row * H + c) = pk;
      if ((tid & 7) == 0) {
        const int kb = c >> 5;
        a.sf[((size_t)(row >> 7) * (H >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] = code;
      }
    }
  }
}

// The last CTA of a call re-arms the completion counter and advances the epoch (every CTA
// read the epoch at its start; the next call starts after this kernel completes).
__device__ __forceinline__ void finish_call(uint32_t* counter, uint32_t* epoch, uint32_t E) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {
      *reinterpret_cast<volatile uint32_t*>(counter) = 0u;
      *reinterpret_cast<volatile uint32_t*>(epoch) = E;
    }
  }
}

__device__ __forceinline__ uint32_t read_epoch(const uint32_t* epoch) {
  return *reinterpret_cast<const volatile uint32_t*>(epoch) + 1u;  // this call's flag value
}

// ---------------------------------------------------------------------------------
// One-shot: CTA = row.  Push lines of the row to every rank's slot [parity][rank][row],
// then sum residual + the W slots in rank order.
__global__ void __launch_bounds__(THREADS, 3) ar_oneshot_kernel(const FusedArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int H = a.hidden, W = a.world, L = H / 4, lpt = L / THREADS;
  const int row = blockIdx.x, tid = threadIdx.x;
  const uint32_t E = read_epoch(a.epoch);
  const int par = E & 1;
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  __shared__ float red[THREADS / 32];
  if (tid == 0) give_up = 0;
  __syncthreads();
  auto slot = [&](int dst_rank, int src) {
    return static_cast<uint4*>(a.part[dst_rank]) + (((size_t)par * W + src) * FAR_ONESHOT_ROWS + row) * L;
  };
  for (int i = 0; i < lpt && !a.pushed; ++i) {
    const int l = tid + i * THREADS;
    const float4 f = local_line(a, row, l);
    const uint32_t d0 = pack_bf16x2(f.x, f.y), d1 = pack_bf16x2(f.z, f.w);
    for (int q = 0; q < W; ++q) st_ll16(slot(q, a.rank) + l, d0, d1, E);
  }
  const __nv_bfloat16* resid = static_cast<const __nv_bfloat16*>(a.residual) + (size_t)row * H;
  const size_t src_stride = (size_t)FAR_ONESHOT_ROWS * L;
  uint2 res[MAX_LPT];
  bool ok = true;
#pragma unroll
  for (int i = 0; i < MAX_LPT; ++i) {
    if (i >= lpt) break;
    const int l = tid + i * THREADS;
    uint4 v[8];
    ok = ok && wait_lines<8>(slot(a.rank, 0) + l, src_stride, W, E, v, budget, a.err, &give_up);
    const uint2 ru = *reinterpret_cast<const uint2*>(resid + 4 * l);
    float4 acc = bf16x4_to_f4(ru.x, ru.y);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q >= W) break;
      const float4 f = bf16x4_to_f4(v[q].x, v[q].z);
      acc.x += f.x;
      acc.y += f.y;
      acc.z += f.z;
      acc.w += f.w;
    }
    res[i] = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
  }
  if (__syncthreads_or(!ok) == 0) finish_row(a, row, lpt, res, red);
  finish_call(a.grid_counter, a.epoch, E);
}

// ---------------------------------------------------------------------------------
// Two-shot with LL lines.  CTA c handles rows c, c + G, ... in every phase on every rank.
//  1. send   : local lines of each row to the row's owner, slot [rank][row - owner_first]
//  2. reduce : the owner sums residual + W slots in rank order, pushes the bf16 result
//              line to every rank's gather buffer
//  3. gather : every rank waits for each row's result lines, then finish_row
// Buffer reuse needs no extra barrier: a rank writes call E+1's lines only after it
// finished call E, and finishing call E required every owner to have read all of call E's
// reduce-scatter slots (an owner sends results only after reading them) and every rank to
// have read call E's results for all rows (its own gather).
__global__ void __launch_bounds__(THREADS, 4) ar_twoshot_kernel(const FusedArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int H = a.hidden, M = a.rows, W = a.world, L = H / 4, lpt = L / THREADS;
  const int tid = threadIdx.x, G = gridDim.x;
  const int per = (M + W - 1) / W;
  const uint32_t E = read_epoch(a.epoch);
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  __shared__ float red[THREADS / 32];
  if (tid == 0) give_up = 0;
  __syncthreads();
  // 1. send (unless the producing GEMM's epilogue already pushed these lines)
  for (int row = blockIdx.x; row < M && !a.pushed; row += G) {
    const int owner = min(row / per, W - 1);
    uint4* dst = static_cast<uint4*>(a.part[owner]) + ((size_t)a.rank * per + (row - owner * per)) * L;
    for (int l = tid; l < L; l += THREADS) {
      const float4 f = local_line(a, row, l);
      st_ll16(dst + l, pack_bf16x2(f.x, f.y), pack_bf16x2(f.z, f.w), E);
    }
  }
  // 2. reduce the owned rows, broadcast the results
  const size_t src_stride = (size_t)per * L;
  for (int row = blockIdx.x; row < M; row += G) {
    const int owner = min(row / per, W - 1);
    if (owner != a.rank) continue;
    const uint4* src = static_cast<const uint4*>(a.part[a.rank]) + (size_t)(row - owner * per) * L;
    const __nv_bfloat16* resid = static_cast<const __nv_bfloat16*>(a.residual) + (size_t)row * H;
    for (int l = tid; l < L; l += THREADS) {
      uint4 v[8];
      if (!wait_lines<8>(src + l, src_stride, W, E, v, budget, a.err, &give_up)) break;
      const uint2 ru = *reinterpret_cast<const uint2*>(resid + 4 * l);
      float4 acc = bf16x4_to_f4(ru.x, ru.y);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (q >= W) break;
        const float4 f = bf16x4_to_f4(v[q].x, v[q].z);
        acc.x += f.x;
        acc.y += f.y;
        acc.z += f.z;
        acc.w += f.w;
      }
      const uint32_t r0 = pack_bf16x2(acc.x, acc.y), r1 = pack_bf16x2(acc.z, acc.w);
      for (int q = 0; q < W; ++q) st_ll16(static_cast<uint4*>(a.out[q]) + (size_t)row * L + l, r0, r1, E);
    }
  }
  // 3. gather + RMSNorm + MXFP8
  for (int row = blockIdx.x; row < M; row += G) {
    const uint4* ag = static_cast<const uint4*>(a.out[a.rank]) + (size_t)row * L;
    uint4 v[MAX_LPT];
    const bool ok = wait_lines<MAX_LPT>(ag + tid, THREADS, lpt, E, v, budget, a.err, &give_up);
    if (__syncthreads_or(!ok)) break;
    uint2 res[MAX_LPT];
#pragma unroll
    for (int i = 0; i < MAX_LPT; ++i) res[i] = make_uint2(v[i].x, v[i].z);
    finish_row(a, row, lpt, res, red);
  }
  finish_call(a.grid_counter, a.epoch, E);
}

// ---------------------------------------------------------------------------------
// NVLS (NVLink SHARP): part, out and flags live in memory bound to one NVSwitch multicast
// object.  CTA c owns rows c, c + G, ... on every rank (G = FAR_CTAS on every call, so
// flag c counts every call):
//  1. this rank's local sums of those rows -> its own part rows (plain local stores)
//  2. barrier: multimem.red.release adds 1 to flag [0][c] of every rank; wait until the
//     local copy reaches world * E
//  3. for this rank's column slice of each row: multimem.ld_reduce (the switch returns
//     the sum over ranks, accumulated in fp32), + residual, rounded to bf16, multimem.st
//     into every rank's out row
//  4. barrier on flag [1][c]; every rank reads its local out rows: finish_row.
// Reuse needs nothing more: a call's part stores follow the previous call's phase-4
// barrier (no rank still reduces the old rows) and its out stores follow this call's
// phase-2 barrier (every rank has finished the previous call: a kernel waits for its
// predecessor before its first access).  Each result element comes from one reduction
// and is broadcast, so every rank holds identical bits.
__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void mm_st_bf16x8(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Every thread's stores of this CTA are published, then one thread adds 1 to flag `slot`
// of every rank through the multicast address and waits (bounded) until its local copy
// reaches `target`.  Returns false for every thread when the wait ran out.
__device__ __forceinline__ bool nvls_barrier(const FusedArArgs& a, int slot, uint32_t target, uint64_t budget) {
  __threadfence_system();
  asm volatile("fence.proxy.alias;" ::: "memory");
  __syncthreads();
  int ok = 1;
  if (threadIdx.x == 0) {
    asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(a.mc_flags + slot), "r"(1u) : "memory");
    ok = wait_flag_sys(a.flags[a.rank] + slot, target, budget, nullptr);
    if (!ok) report_error(a.err, kErrPeerTimeout);
  }
  const bool all_ok = !__syncthreads_or(!ok);
  asm volatile("fence.proxy.alias;" ::: "memory");
  return all_ok;
}

__global__ void __launch_bounds__(THREADS, 4) ar_nvls_kernel(const FusedArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int H = a.hidden, M = a.rows, W = a.world, L = H / 4, lpt = L / THREADS;
  const int tid = threadIdx.x, G = gridDim.x, c = blockIdx.x;
  const uint32_t E = read_epoch(a.epoch);
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ float red[THREADS / 32];
  const int nrows = c < M ? (M - 1 - c) / G + 1 : 0;
  __nv_bfloat16* part = static_cast<__nv_bfloat16*>(a.part[a.rank]);
  // 1. local sums -> own part rows
  for (int k = 0; k < nrows; ++k) {
    const int row = c + k * G;
    for (int l = tid; l < L; l += THREADS) {
      const float4 f = local_line(a, row, l);
      *reinterpret_cast<uint2*>(part + (size_t)row * H + 4 * l) =
          make_uint2(pack_bf16x2(f.x, f.y), pack_bf16x2(f.z, f.w));
    }
  }
  // On a timeout every later phase is skipped (the error word tells the host to reset);
  // the CTA still counts itself in finish_call.
  bool ok = nvls_barrier(a, c, (uint32_t)W * E, budget);
  // 2. switch reduction of this rank's column slice, + residual, broadcast
  const int slice = H / 8 / W;  // 16-byte chunks of the slice
  const int j0 = a.rank * slice;
  for (int it = tid; ok && it < nrows * slice; it += THREADS) {
    const int row = c + (it / slice) * G;
    const size_t off = (size_t)row * H + (size_t)(j0 + it % slice) * 8;  // elements
    const uint4 s = mm_ld_reduce_bf16x8(static_cast<const __nv_bfloat16*>(a.mc_part) + off);
    const uint4 r = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.residual) + off);
    float fs[8], fr[8];
    unpack8(s, fs);
    unpack8(r, fr);
#pragma unroll
    for (int i = 0; i < 8; ++i) fs[i] += fr[i];
    mm_st_bf16x8(static_cast<__nv_bfloat16*>(a.mc_out) + off, pack8(fs));
  }
  ok = ok && nvls_barrier(a, FAR_CTAS + c, (uint32_t)W * E, budget);
  // 3. local result rows -> residual, RMSNorm, MXFP8
  const __nv_bfloat16* out = static_cast<const __nv_bfloat16*>(a.out[a.rank]);
  for (int k = 0; ok && k < nrows; ++k) {
    const int row = c + k * G;
    uint2 res[MAX_LPT];
#pragma unroll
    for (int i = 0; i < MAX_LPT; ++i)
      if (i < lpt) res[i] = ld_ll(reinterpret_cast<const uint2*>(out + (size_t)row * H + 4 * (tid + i * THREADS)));
    finish_row(a, row, lpt, res, red);
  }
  finish_call(a.grid_counter, a.epoch, E);
}

// ---------------------------------------------------------------------------------
// Two-shot with plain bf16 rows (prefill sizes).  Flags: [phase][source][CTA] u32 per rank.
// After a CTA's stores of a phase, every thread fences at system scope, then thread q
// releases flag [phase][rank][c] on rank q; a consumer CTA c acquires the W flags of CTA
// c on every rank before it reads.  Reuse across calls follows the two-shot argument.
template <typename Args>
__device__ __forceinline__ void publish(const Args& a, int phase, uint32_t E) {
  __syncthreads();  // every store of this CTA precedes the fences below
  if (threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + ((size_t)phase * 8 + a.rank) * FAR_CTAS + blockIdx.x, E);
  }
}

template <typename Args>
__device__ __forceinline__ bool await(const Args& a, int phase, uint32_t E, uint64_t budget,
                                      volatile int* give_up) {
  if (threadIdx.x < a.world) {
    const uint32_t* f = a.flags[a.rank] + ((size_t)phase * 8 + threadIdx.x) * FAR_CTAS + blockIdx.x;
    if (!wait_flag_sys(f, E, budget, nullptr)) {
      report_error(a.err, kErrPeerTimeout);
      *give_up = 1;
    }
  }
  __syncthreads();
  return *give_up == 0;
}

__global__ void __launch_bounds__(THREADS, 4) ar_plain_kernel(const FusedArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int H = a.hidden, M = a.rows, W = a.world, L = H / 4, lpt = L / THREADS;
  const int tid = threadIdx.x, G = gridDim.x;
  const int per = (M + W - 1) / W;
  const uint32_t E = read_epoch(a.epoch);
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  __shared__ float red[THREADS / 32];
  if (tid == 0) give_up = 0;
  __syncthreads();
  // 1. send (8 columns per 16-byte store)
  const int L8 = H / 8;
  for (int row = blockIdx.x; row < M; row += G) {
    const int owner = min(row / per, W - 1);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.part[owner]) +
                                          ((size_t)a.rank * per + (row - owner * per)) * H);
    for (int j = tid; j < L8; j += THREADS) {
      const float4 f0 = local_line(a, row, 2 * j), f1 = local_line(a, row, 2 * j + 1);
      dst[j] = make_uint4(pack_bf16x2(f0.x, f0.y), pack_bf16x2(f0.z, f0.w), pack_bf16x2(f1.x, f1.y),
                          pack_bf16x2(f1.z, f1.w));
    }
  }
  publish(a, 0, E);
  // 2. reduce the owned rows, push them to every rank
  if (await(a, 0, E, budget, &give_up)) {
    for (int row = blockIdx.x; row < M; row += G) {
      const int owner = min(row / per, W - 1);
      if (owner != a.rank) continue;
      const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(a.part[a.rank]) + (size_t)(row - owner * per) * H;
      const __nv_bfloat16* resid = static_cast<const __nv_bfloat16*>(a.residual) + (size_t)row * H;
      for (int j = tid; j < L8; j += THREADS) {
        uint4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < W) v[q] = __ldcg(reinterpret_cast<const uint4*>(src + (size_t)q * per * H) + j);
        const uint4 ru = *reinterpret_cast<const uint4*>(resid + 8 * j);
        float4 lo = bf16x4_to_f4(ru.x, ru.y), hi = bf16x4_to_f4(ru.z, ru.w);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q >= W) break;
          const float4 a0 = bf16x4_to_f4(v[q].x, v[q].y), a1 = bf16x4_to_f4(v[q].z, v[q].w);
          lo.x += a0.x;
          lo.y += a0.y;
          lo.z += a0.z;
          lo.w += a0.w;
          hi.x += a1.x;
          hi.y += a1.y;
          hi.z += a1.z;
          hi.w += a1.w;
        }
        const uint4 r = make_uint4(pack_bf16x2(lo.x, lo.y), pack_bf16x2(lo.z, lo.w), pack_bf16x2(hi.x, hi.y),
                                   pack_bf16x2(hi.z, hi.w));
        for (int q = 0; q < W; ++q)
          reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out[q]) + (size_t)row * H)[j] = r;
      }
    }
  }
  publish(a, 1, E);
  // 3. gather + RMSNorm + MXFP8
  if (await(a, 1, E, budget, &give_up)) {
    for (int row = blockIdx.x; row < M; row += G) {
      const uint2* ag = reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.out[a.rank]) +
                                                       (size_t)row * H);
      uint2 res[MAX_LPT];
#pragma unroll
      for (int i = 0; i < MAX_LPT; ++i)
        if (i < lpt) res[i] = __ldcg(ag + tid + i * THREADS);
      finish_row(a, row, lpt, res, red);
    }
  }
  finish_call(a.grid_counter, a.epoch, E);
}

// ---------------------------------------------------------------------------------
// One-shot fp32 sum: line i = elements (2i, 2i+1); each thread pushes its lines to every
// rank, then sums exactly the lines it pushed in rank order (so it only waits for peers).
__global__ void __launch_bounds__(THREADS, 4) allreduce_sum_f32_kernel(const SumArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int W = a.world;
  const uint32_t E = read_epoch(a.epoch);
  const int par = E & 1;
  const size_t n = (size_t)a.rows * a.cols / 2;
  const size_t stride = (size_t)a.max_rows * a.cols / 2;
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  if (threadIdx.x == 0) give_up = 0;
  __syncthreads();
  const size_t step = (size_t)gridDim.x * THREADS;
  const float2* data2 = reinterpret_cast<const float2*>(a.data);
  for (size_t i = (size_t)blockIdx.x * THREADS + threadIdx.x; i < n; i += step) {
    const float2 v = data2[i];
    for (int q = 0; q < W; ++q)
      st_ll16(static_cast<uint4*>(a.buf[q]) + ((size_t)par * W + a.rank) * stride + i, __float_as_uint(v.x),
              __float_as_uint(v.y), E);
  }
  for (size_t i = (size_t)blockIdx.x * THREADS + threadIdx.x; i < n; i += step) {
    uint4 v[8];
    if (!wait_lines<8>(static_cast<const uint4*>(a.buf[a.rank]) + (size_t)par * W * stride + i, stride, W, E, v,
                       budget, a.err, &give_up))
      break;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q >= W) break;
      s0 += __uint_as_float(v[q].x);
      s1 += __uint_as_float(v[q].z);
    }
    reinterpret_cast<float2*>(a.data)[i] = make_float2(s0, s1);
  }
  finish_call(a.grid_counter, a.epoch, E);
}

// ---------------------------------------------------------------------------------
// Plain two-shot fp32 sum (rows above the one-shot capacity): the FAR_PLAIN data flow on
// fp32 rows without the norm.  Owners sum the W contributions in rank order, so every
// rank ends with the same bits.
__global__ void __launch_bounds__(THREADS, 4) allreduce_sum_f32_plain_kernel(const SumArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int M = a.rows, W = a.world, C4 = a.cols / 4, tid = threadIdx.x, G = gridDim.x;
  const int per = (M + W - 1) / W;
  const uint32_t E = read_epoch(a.epoch);
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  if (tid == 0) give_up = 0;
  __syncthreads();
  const float4* src4 = reinterpret_cast<const float4*>(a.data);
  for (int row = blockIdx.x; row < M; row += G) {
    const int owner = min(row / per, W - 1);
    float4* dst = static_cast<float4*>(a.part[owner]) + ((size_t)a.rank * per + (row - owner * per)) * C4;
    for (int j = tid; j < C4; j += THREADS) dst[j] = src4[(size_t)row * C4 + j];
  }
  publish(a, 0, E);
  if (await(a, 0, E, budget, &give_up)) {
    for (int row = blockIdx.x; row < M; row += G) {
      const int owner = min(row / per, W - 1);
      if (owner != a.rank) continue;
      const float4* part = static_cast<const float4*>(a.part[a.rank]) + (size_t)(row - owner * per) * C4;
      for (int j = tid; j < C4; j += THREADS) {
        float4 acc = __ldcg(part + j);
        for (int q = 1; q < W; ++q) {
          const float4 v = __ldcg(part + (size_t)q * per * C4 + j);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        for (int q = 0; q < W; ++q) (static_cast<float4*>(a.out[q]) + (size_t)row * C4)[j] = acc;
      }
    }
  }
  publish(a, 1, E);
  if (await(a, 1, E, budget, &give_up)) {
    float4* dst4 = reinterpret_cast<float4*>(a.data);
    for (int row = blockIdx.x; row < M; row += G) {
      const float4* res = static_cast<const float4*>(a.out[a.rank]) + (size_t)row * C4;
      for (int j = tid; j < C4; j += THREADS) dst4[(size_t)row * C4 + j] = __ldcg(res + j);
    }
  }
  finish_call(a.grid_counter, a.epoch, E);
}

// ---------------------------------------------------------------------------------
// Global argmax: one warp per row reduces the row's tile keys, rebases the id to the
// global vocabulary, and lane 0 pushes the key as one LL line to every rank's slot
// [parity][rank][row]; then the warp waits for the W lines of the row and max-reduces.
constexpr int ARGMAX_WARPS = 8;

__global__ void __launch_bounds__(ARGMAX_WARPS * 32) allreduce_argmax_kernel(const ArgmaxArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int W = a.world;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * ARGMAX_WARPS + warp;
  const uint32_t E = read_epoch(a.epoch);
  const int par = E & 1;
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  if (threadIdx.x == 0) give_up = 0;
  __syncthreads();
  if (row < a.rows) {
    unsigned long long best = 0;
    for (int t = lane; t < a.tiles; t += 32) {
      const unsigned long long k = a.tile_keys[(size_t)row * a.tiles + t];
      best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffff, best, o);
      best = other > best ? other : best;
    }
    // Rebase the local id (the logit half of the key is unchanged).
    const int gid = unpack_argmax_id(best) + a.id_offset;
    best = (best & 0xFFFFFFFF00000000ull) | static_cast<uint32_t>(~gid);
    const size_t src_stride = (size_t)a.max_rows;
    if (lane < W)
      st_ll16(static_cast<uint4*>(a.lines[lane]) + ((size_t)par * W + a.rank) * src_stride + row,
              static_cast<uint32_t>(best), static_cast<uint32_t>(best >> 32), E);
    unsigned long long g = 0;
    if (lane < W) {
      uint4 v[1];
      if (wait_lines<1>(static_cast<const uint4*>(a.lines[a.rank]) + ((size_t)par * W + lane) * src_stride + row, 0,
                        1, E, v, budget, a.err, &give_up))
        g = (static_cast<unsigned long long>(v[0].z) << 32) | v[0].x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffff, g, o);
      g = other > g ? other : g;
    }
    if (lane == 0) {
      if (a.out_ids) a.out_ids[row] = unpack_argmax_id(g);
      if (a.out_vals) a.out_vals[row] = unpack_argmax_value(g);
    }
  }
  finish_call(a.grid_counter, a.epoch, E);
}

}  // namespace coll
}  // namespace zs

// ----------------------------------------------------------------------------------- host
extern "C" int zs_fused_allreduce_norm(const FusedArArgs* args, cudaStream_t stream) {
  using namespace zs::coll;
  const FusedArArgs& a = *args;
  if (a.world < 1 || a.world > 8 || a.hidden % (THREADS * 4) != 0 || a.hidden > THREADS * 4 * MAX_LPT) return -1;
  if (a.protocol == FAR_NVLS) {
    if (a.rank < 0 || a.rank >= a.world || a.part[a.rank] == nullptr || a.out[a.rank] == nullptr ||
        a.flags[a.rank] == nullptr || a.mc_part == nullptr || a.mc_out == nullptr || a.mc_flags == nullptr ||
        a.pushed || (a.hidden / 8) % a.world != 0)
      return -1;
  } else {
    for (int r = 0; r < a.world; ++r)
      if (a.part[r] == nullptr || (a.protocol != FAR_ONESHOT && a.out[r] == nullptr) ||
          (a.protocol == FAR_PLAIN && a.flags[r] == nullptr))
        return -1;
  }
  if (a.rows <= 0) return 0;
  if (a.pushed && a.protocol == FAR_PLAIN) return -1;
  cudaError_t e;
  if (a.protocol == FAR_ONESHOT) {
    if (a.rows > FAR_ONESHOT_ROWS) return -1;
    e = zs_launch(ar_oneshot_kernel, a.rows, THREADS, 0, stream, a);
  } else if (a.protocol == FAR_TWOSHOT) {
    e = zs_launch(ar_twoshot_kernel, FAR_CTAS, THREADS, 0, stream, a);
  } else if (a.protocol == FAR_PLAIN) {
    e = zs_launch(ar_plain_kernel, FAR_CTAS, THREADS, 0, stream, a);
  } else if (a.protocol == FAR_NVLS) {
    e = zs_launch(ar_nvls_kernel, FAR_CTAS, THREADS, 0, stream, a);  // every CTA index on every call
  } else {
    return -1;
  }
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int zs_allreduce_argmax(const ArgmaxArArgs* args, cudaStream_t stream) {
  using namespace zs::coll;
  const ArgmaxArArgs& a = *args;
  if (a.world < 1 || a.world > 8 || a.rows > a.max_rows || a.tiles <= 0) return -1;
  for (int r = 0; r < a.world; ++r)
    if (a.lines[r] == nullptr) return -1;
  if (a.rows <= 0) return 0;
  const cudaError_t e =
      zs_launch(allreduce_argmax_kernel, (a.rows + ARGMAX_WARPS - 1) / ARGMAX_WARPS, ARGMAX_WARPS * 32, 0, stream, a);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int zs_allreduce_sum_f32(const SumArArgs* args, cudaStream_t stream) {
  using namespace zs::coll;
  const SumArArgs& a = *args;
  if (a.plain) {
    if (a.world < 1 || a.world > 8 || a.rows < 0 || a.cols <= 0 || (a.cols & 3)) return -1;
    for (int r = 0; r < a.world; ++r)
      if (a.part[r] == nullptr || a.out[r] == nullptr || a.flags[r] == nullptr) return -1;
    if (a.rows == 0) return 0;
    const cudaError_t e = zs_launch(allreduce_sum_f32_plain_kernel, FAR_CTAS, THREADS, 0, stream, a);
    return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
  if (a.world < 1 || a.world > 8 || a.rows < 0 || a.rows > a.max_rows || a.cols <= 0 || (a.cols & 1)) return -1;
  for (int r = 0; r < a.world; ++r)
    if (a.buf[r] == nullptr) return -1;
  if (a.rows == 0) return 0;
  const cudaError_t e = zs_launch(allreduce_sum_f32_kernel, SUM_CTAS, THREADS, 0, stream, a);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Symmetric memory helpers: raw cudaMalloc blocks shared through CUDA IPC.
extern "C" int zs_symm_alloc(size_t bytes, void** ptr) {
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return -1;
  return cudaMemset(*ptr, 0, bytes) == cudaSuccess ? 0 : -2;
}
extern "C" int zs_symm_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? 0 : -1; }
extern "C" int zs_ipc_handle(void* ptr, void* handle_out /* 64 bytes */) {
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return -1;
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}
extern "C" int zs_ipc_open(const void* handle, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? 0 : -1;
}
extern "C" int zs_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : -1; }

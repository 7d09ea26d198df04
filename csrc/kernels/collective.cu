// Tensor-parallel collectives fused with their consumers, over NVLink peer memory.
//
// Symmetric memory: every rank allocates the same buffers with cudaMalloc and maps its
// peers' copies through CUDA IPC (cudaIpcOpenMemHandle), so a kernel on rank r can load
// from and store to rank q's buffer directly over NVLink / NVSwitch.  No host memory
// and no library collective sits on the data path.
//
// fused_allreduce_norm (one cooperative launch): push-based two-shot all-reduce of the
// row-parallel partial sums with flag-in-data words, fused with the residual add, RMSNorm
// and MXFP8 quantization (details at the kernel).  Every word carries the call's epoch
// (a counter in device memory advanced by the kernel itself), so there is no separate
// barrier round trip and the kernel stays CUDA-graph safe.
//
// allreduce_argmax: per-row packed (logit, ~id) keys of each rank's vocab shard are
// exchanged the same way and max-reduced, giving the global greedy token on every rank.
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

using namespace peer;


// Local contribution to word w (elements 2w, 2w+1) of `row`: the rank's terms summed in
// term order, rounded to bf16 (what the other ranks receive).
__device__ __forceinline__ uint32_t local_word(const FusedArArgs& a, int row, int w) {
  float s0 = 0.f, s1 = 0.f;
  const int c = 2 * w;
  for (int t = 0; t < a.n_terms; ++t) {
    long long off = row * a.row_stride + t * a.term_stride + c;
    float sc = 1.f;
    if (a.term_index != nullptr) {  // gathered term; negative = not produced on this rank
      const int src = a.term_index[row * a.n_terms + t];
      if (src < 0) continue;
      off = (long long)src * a.row_stride + c;
    }
    if (a.term_scale != nullptr) sc = a.term_scale[row * a.n_terms + t];
    if (a.delta_f32) {
      const float2 v = *reinterpret_cast<const float2*>(static_cast<const float*>(a.delta) + off);
      s0 += sc * v.x;
      s1 += sc * v.y;
    } else {
      const float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(static_cast<const __nv_bfloat16*>(a.delta) + off));
      s0 += sc * v.x;
      s1 += sc * v.y;
    }
  }
  return pack_bf16x2(s0, s1);
}

// Push-based two-shot all-reduce with flag-in-data words (no grid barrier, no remote loads):
//  1. send   : every rank pushes its bf16 local sum of each row to the row's owner
//              (rs buffer slot [sender][row - owner_first_row])
//  2. reduce : the owner waits for the W contributions of its rows, adds residual + the
//              contributions in rank order (identical on every rank) and pushes the bf16
//              result to every rank's ag buffer
//  3. gather : every rank waits for each row's result, writes it to its residual stream
//              and applies RMSNorm + MXFP8 quantization
// CTA c handles rows c, c+G, ... in all three phases on every rank, so a CTA only waits for
// words that other CTAs (same index, other ranks) produce before they wait themselves.
// Buffers are reused across calls without extra barriers: a rank writes call E+1's words
// only after it finished call E, which needed every peer's call-E words it is about to
// overwrite to have been consumed (an owner sends its results only after reading all
// contributions; a sender starts the next call only after reading all results).
__global__ void __launch_bounds__(THREADS) fused_allreduce_norm_kernel(const FusedArArgs a) {
  const int H = a.hidden, M = a.rows, W = a.world;
  const int words = H / 2;
  const int tid = threadIdx.x;
  const uint32_t E = *reinterpret_cast<volatile uint32_t*>(a.epoch) + 1;  // this call's flag value (never 0)
  const int G = gridDim.x;
  const int per = (M + W - 1) / W;
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  if (tid == 0) give_up = 0;
  __syncthreads();

  // 1. send local sums to the owners
  for (int row = blockIdx.x; row < M; row += G) {
    const int owner = min(row / per, W - 1);
    uint2* dst = static_cast<uint2*>(a.part[owner]) + ((size_t)a.rank * per + (row - owner * per)) * words;
    for (int w = tid; w < words; w += THREADS) st_ll(dst + w, local_word(a, row, w), E);
  }
  // 2. reduce the owned rows and broadcast them
  const __nv_bfloat16* resid = static_cast<const __nv_bfloat16*>(a.residual);
  for (int row = blockIdx.x; row < M; row += G) {
    const int owner = min(row / per, W - 1);
    if (owner != a.rank) continue;
    const uint2* src = static_cast<const uint2*>(a.part[a.rank]) + (size_t)(row - owner * per) * words;
    for (int w = tid; w < words; w += THREADS) {
      float2 acc = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(resid + (size_t)row * H + 2 * w));
      for (int q = 0; q < W; ++q) {
        const float2 v = unpack_bf16x2(wait_ll(src + (size_t)q * per * words + w, E, budget, a.err, &give_up));
        acc.x += v.x;
        acc.y += v.y;
      }
      const uint32_t res = pack_bf16x2(acc.x, acc.y);
      for (int q = 0; q < W; ++q) st_ll(static_cast<uint2*>(a.out[q]) + (size_t)row * words + w, res, E);
    }
  }
  // 3. gather every row, then RMSNorm + MXFP8
  __shared__ float red[THREADS / 32];
  __nv_bfloat16* res_out = static_cast<__nv_bfloat16*>(a.residual);
  const __nv_bfloat16* wgt = static_cast<const __nv_bfloat16*>(a.weight);
  const uint2* ag = static_cast<const uint2*>(a.out[a.rank]);
  for (int row = blockIdx.x; row < M; row += G) {
    float x[4][8];
    float ss = 0.f;
    const int iters = H / (THREADS * 8);
    for (int it = 0; it < iters; ++it) {
      const int c = (it * THREADS + tid) * 8;
      uint32_t u[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        u[j] = wait_ll(ag + (size_t)row * words + c / 2 + j, E, budget, a.err, &give_up);
        const float2 f = unpack_bf16x2(u[j]);
        x[it][2 * j] = f.x;
        x[it][2 * j + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
      *reinterpret_cast<uint4*>(res_out + (size_t)row * H + c) = make_uint4(u[0], u[1], u[2], u[3]);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) tot += red[i];
    __syncthreads();
    const float rstd = rsqrtf(tot / H + a.eps);
    for (int it = 0; it < iters; ++it) {
      const int c = (it * THREADS + tid) * 8;
      float w8[8], y[8];
      unpack8(*reinterpret_cast<const uint4*>(wgt + c), w8);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = x[it][j] * rstd * (w8[j] + a.w_offset);
      if (a.normed) *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.normed) + (size_t)row * H + c) = pack8(y);
      if (a.q) {
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(y[j]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 2));
        const uint8_t code = mx_scale_e8m0(amax);
        const float inv = mx_inv_scale(code);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lo |= uint32_t(f32_to_e4m3(y[j] * inv)) << (8 * j);
          hi |= uint32_t(f32_to_e4m3(y[4 + j] * inv)) << (8 * j);
        }
        *reinterpret_cast<uint2*>(a.q + (size_t)row * H + c) = make_uint2(lo, hi);
        if ((tid & 3) == 0) {
          const int kb = c >> 5;
          a.sf[((size_t)(row >> 7) * (H >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] = code;
        }
      }
    }
  }
  // The last CTA to finish advances the epoch (every CTA has read it by then).
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(a.grid_counter, 1u) + 1;
    if (done % (uint32_t)G == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch) = E;
  }
}

// Global argmax over vocab shards: keys[r] = per-row best packed key of rank r's shard
// (ids already global).  Every rank max-reduces all W keys per row.
__global__ void allreduce_argmax_kernel(const ArgmaxArArgs a) {
  const uint32_t E = *reinterpret_cast<volatile uint32_t*>(a.epoch);
  const int tid = threadIdx.x;
  // Publish this rank's keys (already in its symmetric buffer), then barrier.
  __shared__ int ok;
  __threadfence_system();  // keys written by rebase_keys_kernel before the release
  if (tid < a.world) st_release_sys(a.flags[tid] + 16 + a.rank, E + 1);
  if (tid == 0) {
    ok = 1;
    for (int r = 0; r < a.world && ok; ++r) {
      if (!wait_flag_sys(a.flags[a.rank] + 16 + r, E + 1, limit_ns(a.timeout_ms), nullptr)) {
        ok = 0;
        report_error(a.err, kErrPeerTimeout);
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  for (int row = tid; row < a.rows; row += blockDim.x) {
    unsigned long long best = 0;
    for (int r = 0; r < a.world; ++r) {
      const unsigned long long* kp = static_cast<const unsigned long long*>(a.keys[r]) + row;
      unsigned long long k;
      asm volatile("ld.global.cv.u64 %0, [%1];" : "=l"(k) : "l"(kp) : "memory");
      best = k > best ? k : best;
    }
    if (a.out_ids) a.out_ids[row] = unpack_argmax_id(best);
    if (a.out_vals) a.out_vals[row] = unpack_argmax_value(best);
  }
  __syncthreads();
  // Second barrier: no rank may overwrite its keys before every peer has read them.
  if (tid < a.world) st_release_sys(a.flags[tid] + 24 + a.rank, E + 1);
  if (tid == 0) {
    for (int r = 0; r < a.world; ++r)
      if (!wait_flag_sys(a.flags[a.rank] + 24 + r, E + 1, limit_ns(a.timeout_ms), nullptr))
        report_error(a.err, kErrPeerTimeout);
    *reinterpret_cast<volatile uint32_t*>(a.epoch) = E + 1;
  }
}

// Rebase per-row local argmax keys to global ids and store them in the symmetric
// key buffer of this rank.
__global__ void rebase_keys_kernel(const unsigned long long* __restrict__ local, int rows, int id_offset,
                                   unsigned long long* __restrict__ out) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const unsigned long long k = local[row];
  const int lid = unpack_argmax_id(k);
  out[row] = (k & 0xFFFFFFFF00000000ull) | static_cast<uint32_t>(~(lid + id_offset));
}

}  // namespace coll
}  // namespace zs

// ----------------------------------------------------------------------------------- host
extern "C" int zs_fused_allreduce_norm(const FusedArArgs* args, cudaStream_t stream) {
  const FusedArArgs& a = *args;
  if (a.world < 1 || a.world > 8 || a.hidden % (zs::coll::THREADS * 8) != 0 || a.hidden > zs::coll::THREADS * 8 * 4)
    return -1;
  if (a.rows <= 0) return 0;
  // Cooperative launch: the grid barrier needs all FAR_CTAS CTAs co-resident.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(FAR_CTAS);
  cfg.blockDim = dim3(zs::coll::THREADS);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, zs::coll::fused_allreduce_norm_kernel, a) == cudaSuccess ? 0 : -2;
}

extern "C" int zs_allreduce_argmax(const ArgmaxArArgs* args, const unsigned long long* local_keys, int id_offset,
                                   cudaStream_t stream) {
  const ArgmaxArArgs& a = *args;
  if (a.world < 1 || a.world > 8) return -1;
  if (a.rows <= 0) return 0;
  zs::coll::rebase_keys_kernel<<<(a.rows + 255) / 256, 256, 0, stream>>>(
      local_keys, a.rows, id_offset, static_cast<unsigned long long*>(const_cast<void*>(a.keys[a.rank])));
  zs::coll::allreduce_argmax_kernel<<<1, 256, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
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

// Tensor-parallel collectives fused with their consumers, over NVLink peer memory.
//
// Symmetric memory: every rank allocates the same buffers with cudaMalloc and maps its
// peers' copies through CUDA IPC (cudaIpcOpenMemHandle), so a kernel on rank r can load
// from and store to rank q's buffer directly over NVLink / NVSwitch.  No host memory
// and no library collective sits on the data path.
//
// fused_allreduce_norm (one persistent kernel, grid of FAR_CTAS co-resident CTAs):
//   1. local term sum   : part[r][row] = sum of this rank's partial terms (f32 split-K
//                         partials or bf16 MoE pair rows), written to symmetric memory
//   2. cross-rank barrier "ready" (release stores into every peer's flag word, acquire
//                         spins on the local flags; all waits bounded)
//   3. reduce-scatter   : rank r owns rows [r*M/W, (r+1)*M/W); for them it adds
//                         residual + part[0] + ... + part[W-1] in rank order (so the
//                         result is bit-identical whichever rank computes it), rounds to
//                         bf16 and writes out[r][row]
//   4. cross-rank barrier "reduced"
//   5. all-gather + norm: every rank copies each row from its owner's out buffer into
//                         its residual stream, then RMSNorm + MXFP8 quantize locally
// A grid-wide barrier (atomic counter, bounded spin) separates the phases inside a rank.
// Phase-3 reads of part[] finish before barrier 4 and phase-5 reads of out[] finish
// before the next call's barrier 2, so no buffer is overwritten while a peer reads it.
// An epoch counter in device memory (same sequence on every rank, advanced by the
// kernel itself) makes flag values monotonic and keeps the kernel CUDA-graph safe.
//
// allreduce_argmax: per-row packed (logit, ~id) keys of each rank's vocab shard are
// exchanged the same way and max-reduced, giving the global greedy token on every rank.
//
// Reference parity: replaces worker/zstep_worker/kernels_sm120/csrc/shm_allreduce_kernels.cu
// (shm_v5 all-reduce :472, fused AR + add + RMSNorm :1376, spin-wait with abort :31-83)
// and the TP=8 argmax exchange (csrc/qwen35_ops_kernels.cu:202).
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace coll {

constexpr int THREADS = 256;

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

// Grid-wide barrier for a persistent grid; `target` grows monotonically across calls.
__device__ __forceinline__ bool grid_sync(uint32_t* counter, uint32_t target, uint64_t budget_ns, int* err) {
  __syncthreads();
  __shared__ int ok;
  if (threadIdx.x == 0) {
    __threadfence_system();
    atomicAdd(counter, 1u);
    ok = 0;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
      if ((int)(ld_acquire_gpu(counter) - target) >= 0) {
        ok = 1;
        break;
      }
      if (i > 32) {
        __nanosleep(32);
        if ((i & 255) == 0 && globaltimer_ns() - t0 > budget_ns) break;
      }
    }
    if (!ok) report_error(err, kErrPeerTimeout);
  }
  __syncthreads();
  return ok != 0;
}

// Cross-rank barrier: CTA 0 releases `value` into slot `rank` of every peer's flag
// array; every CTA then waits until all `world` slots of its local array reach it.
__device__ __forceinline__ bool rank_barrier(const FusedArArgs& a, int phase, uint32_t value) {
  __shared__ int ok;
  if (blockIdx.x == 0 && threadIdx.x < a.world)
    st_release_sys(a.flags[threadIdx.x] + phase * 8 + a.rank, value);
  if (threadIdx.x == 0) {
    ok = 1;
    const uint32_t* mine = a.flags[a.rank] + phase * 8;
    for (int r = 0; r < a.world && ok; ++r) {
      if (!wait_flag_sys(mine + r, value, limit_ns(a.timeout_ms), a.abort_word)) {
        ok = 0;
        report_error(a.err, kErrPeerTimeout);
      }
    }
  }
  __syncthreads();
  return ok != 0;
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

__global__ void __launch_bounds__(THREADS) fused_allreduce_norm_kernel(const FusedArArgs a) {
  const int H = a.hidden, M = a.rows, W = a.world;
  const int tid = threadIdx.x;
  const uint32_t E = *reinterpret_cast<volatile uint32_t*>(a.epoch);
  const uint32_t G = gridDim.x;
  const int chunks = H / 8;  // 16-byte chunks per row

  // 1. local term sum -> part[rank] (bf16)
  __nv_bfloat16* my_part = static_cast<__nv_bfloat16*>(a.part[a.rank]);
  for (long long idx = (long long)blockIdx.x * THREADS + tid; idx < (long long)M * chunks; idx += (long long)G * THREADS) {
    const int row = int(idx / chunks), c = int(idx % chunks) * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
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
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.delta) + off);
        const float4 x0 = p[0], x1 = p[1];
        acc[0] += sc * x0.x; acc[1] += sc * x0.y; acc[2] += sc * x0.z; acc[3] += sc * x0.w;
        acc[4] += sc * x1.x; acc[5] += sc * x1.y; acc[6] += sc * x1.z; acc[7] += sc * x1.w;
      } else {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.delta) + off), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += sc * f[j];
      }
    }
    *reinterpret_cast<uint4*>(my_part + (size_t)row * H + c) = pack8(acc);
  }
  // Two grid barriers per call: the counter reaches 2*G*(E+1) when call E completes.
  if (!grid_sync(a.grid_counter, (E * 2 + 1) * G, limit_ns(a.timeout_ms), a.err)) return;
  if (blockIdx.x == 0 && tid == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch) = E + 1;  // everyone has read E
  if (!rank_barrier(a, 0, E + 1)) return;

  // 3. reduce-scatter of owned rows: out[rank][row] = bf16(residual + sum_r part[r])
  const int per = (M + W - 1) / W;
  const int r0 = a.rank * per, r1 = min(M, r0 + per);
  __nv_bfloat16* my_out = static_cast<__nv_bfloat16*>(a.out[a.rank]);
  const __nv_bfloat16* resid = static_cast<const __nv_bfloat16*>(a.residual);
  for (long long idx = (long long)blockIdx.x * THREADS + tid; idx < (long long)(r1 - r0) * chunks;
       idx += (long long)G * THREADS) {
    const int row = r0 + int(idx / chunks), c = int(idx % chunks) * 8;
    const size_t off = (size_t)row * H + c;
    float acc[8], f[8];
    unpack8(*reinterpret_cast<const uint4*>(resid + off), acc);
    for (int r = 0; r < W; ++r) {
      unpack8(ld_cv_v4(static_cast<const __nv_bfloat16*>(a.part[r]) + off), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    *reinterpret_cast<uint4*>(my_out + off) = pack8(acc);
  }
  if (!grid_sync(a.grid_counter, (E * 2 + 2) * G, limit_ns(a.timeout_ms), a.err)) return;
  if (!rank_barrier(a, 1, E + 1)) return;

  // 5. all-gather rows into the residual stream, then RMSNorm + MXFP8 quantization.
  __shared__ float red[THREADS / 32];
  __nv_bfloat16* res_out = static_cast<__nv_bfloat16*>(a.residual);
  const __nv_bfloat16* wgt = static_cast<const __nv_bfloat16*>(a.weight);
  for (int row = blockIdx.x; row < M; row += G) {
    const int owner = min(row / per, W - 1);
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(a.out[owner]) + (size_t)row * H;
    float x[4][8];
    float ss = 0.f;
    const int iters = H / (THREADS * 8);
    for (int it = 0; it < iters; ++it) {
      const int c = (it * THREADS + tid) * 8;
      const uint4 u = ld_cv_v4(src + c);  // written this call by another SM or GPU
      *reinterpret_cast<uint4*>(res_out + (size_t)row * H + c) = u;
      unpack8(u, x[it]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += x[it][j] * x[it][j];
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
      float w[8], y[8];
      unpack8(*reinterpret_cast<const uint4*>(wgt + c), w);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = x[it][j] * rstd * (w[j] + a.w_offset);
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

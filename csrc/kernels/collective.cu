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
// fused_allreduce_norm_small (rows <= 8): one-shot instead of two-shot (one NVLink hop),
// one 8-CTA cluster per row splitting its columns; the RMSNorm sum of squares is combined
// through distributed shared memory.
//
// allreduce_argmax: per-row packed (logit, ~id) keys of each rank's vocab shard are
// exchanged the same way and max-reduced, giving the global greedy token on every rank.
//
// allreduce_sum_f32: one-shot in-place fp32 sum (the mHC model's sublayer outputs).
//
// Reference parity: replaces worker/zstep_worker/kernels_sm120/csrc/shm_allreduce_kernels.cu
// (shm_v5 all-reduce :472, fused AR + add + RMSNorm :1376, spin-wait with abort :31-83)
// and the TP=8 argmax exchange (csrc/qwen35_ops_kernels.cu:202).
#include <cooperative_groups.h>

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

// One-shot fused all-reduce for rows <= FAR_SMALL_ROWS.  Cluster = one row; CTA `part`
// owns words [part * cw, (part + 1) * cw) of it.  Every rank pushes its local words of
// the slice to every rank (parity E & 1 of the one-shot buffer, so call E+1 never
// overwrites words a slower rank still waits for in call E: a rank starts call E+2 only
// after every rank finished pushing call E+1, i.e. finished reading call E), then sums
// residual + all ranks' words in rank order, like the two-shot owner does.
constexpr int SMALL_CTAS = 8;

__global__ void __cluster_dims__(SMALL_CTAS, 1, 1) __launch_bounds__(THREADS)
    fused_allreduce_norm_small_kernel(const FusedArArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int H = a.hidden, W = a.world;
  const int words = H / 2, cw = words / SMALL_CTAS;
  const int row = blockIdx.x / SMALL_CTAS;
  const int part = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31;
  const uint32_t E = *reinterpret_cast<volatile uint32_t*>(a.epoch) + 1;
  const int par = E & 1;
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  __shared__ float red[THREADS / 32];
  __shared__ float cta_ss, tot_ss;
  if (tid == 0) give_up = 0;
  __syncthreads();
  // The grid always has FAR_SMALL_ROWS clusters (a fixed CTA count keeps the completion
  // counter a multiple of the grid); clusters past `rows` only count themselves.
  if (row >= a.rows) {
    if (tid == 0) {
      const uint32_t done = atomicAdd(a.grid_counter, 1u) + 1;
      if (done % gridDim.x == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch) = E;
    }
    return;
  }
  auto slot = [&](int q, int src, int w) {
    return static_cast<uint2*>(a.oneshot[q]) + ((((size_t)par * W + src) * FAR_SMALL_ROWS + row) * words + w);
  };
  // 1. push
  for (int w = part * cw + tid; w < (part + 1) * cw; w += THREADS) {
    const uint32_t v = local_word(a, row, w);
    for (int q = 0; q < W; ++q) st_ll(slot(q, a.rank, w), v, E);
  }
  // 2. reduce (residual first, then ranks in order), write the residual
  constexpr int MAXW = 4;  // words per thread: hidden <= 8 * 2 * THREADS * MAXW
  float2 x[MAXW];
  float ss = 0.f;
  __nv_bfloat16* res = static_cast<__nv_bfloat16*>(a.residual);
#pragma unroll
  for (int i = 0; i < MAXW; ++i) {
    x[i] = make_float2(0.f, 0.f);
    const int w = part * cw + tid + i * THREADS;
    if (w >= (part + 1) * cw) continue;
    float2 acc = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(res + (size_t)row * H + 2 * w));
    for (int q = 0; q < W; ++q) {
      const float2 v = unpack_bf16x2(wait_ll(slot(a.rank, q, w), E, budget, a.err, &give_up));
      acc.x += v.x;
      acc.y += v.y;
    }
    const uint32_t r = pack_bf16x2(acc.x, acc.y);
    *reinterpret_cast<uint32_t*>(res + (size_t)row * H + 2 * w) = r;
    x[i] = unpack_bf16x2(r);
    ss += x[i].x * x[i].x + x[i].y * x[i].y;
  }
  // 3. row sum of squares: CTA partials exchanged through distributed shared memory
  ss = warp_sum(ss);
  if (lane == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) t += red[i];
    cta_ss = t;
  }
  cluster.sync();
  if (tid == 0) {
    float t = 0.f;
    for (int r = 0; r < SMALL_CTAS; ++r) t += *cluster.map_shared_rank(&cta_ss, r);
    tot_ss = t;
  }
  cluster.sync();  // no CTA leaves while a peer may still read its cta_ss
  const float rstd = rsqrtf(tot_ss / H + a.eps);
  // 4. RMSNorm + MXFP8 of the slice (16 consecutive threads = one 32-column block)
  const __nv_bfloat16* wgt = static_cast<const __nv_bfloat16*>(a.weight);
#pragma unroll
  for (int i = 0; i < MAXW; ++i) {
    const int w = part * cw + tid + i * THREADS;
    if (part * cw + (tid & ~15) + i * THREADS >= (part + 1) * cw) continue;  // whole block outside
    const bool in = w < (part + 1) * cw;
    const int c = 2 * w;
    float y0 = 0.f, y1 = 0.f;
    if (in) {
      const float2 wv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(wgt + c));
      y0 = x[i].x * rstd * (wv.x + a.w_offset);
      y1 = x[i].y * rstd * (wv.y + a.w_offset);
      if (a.normed) *reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(a.normed) + (size_t)row * H + c) =
          pack_bf16x2(y0, y1);
    }
    if (a.q) {
      float amax = fmaxf(fabsf(y0), fabsf(y1));
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, o));
      const uint8_t code = mx_scale_e8m0(amax);
      const float inv = mx_inv_scale(code);
      if (in) {
        const uint16_t pk = uint16_t(f32_to_e4m3(y0 * inv)) | (uint16_t(f32_to_e4m3(y1 * inv)) << 8);
        *reinterpret_cast<uint16_t*>(a.q + (size_t)row * H + c) = pk;
        if ((tid & 15) == 0) {
          const int kb = c >> 5;
          a.sf[((size_t)(row >> 7) * (H >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] = code;
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(a.grid_counter, 1u) + 1;
    if (done % gridDim.x == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch) = E;
  }
}

// One-shot fp32 sum: each thread pushes its elements to every rank, then sums exactly the
// elements it pushed, so a thread only ever waits for peers.
__global__ void __launch_bounds__(THREADS) allreduce_sum_f32_kernel(const SumArArgs a) {
  const int W = a.world;
  const uint32_t E = *reinterpret_cast<volatile uint32_t*>(a.epoch) + 1;
  const int par = E & 1;
  const size_t n = (size_t)a.rows * a.cols;
  const size_t stride = (size_t)a.max_rows * a.cols;
  const uint64_t budget = limit_ns(a.timeout_ms);
  __shared__ int give_up;
  if (threadIdx.x == 0) give_up = 0;
  __syncthreads();
  const size_t step = (size_t)gridDim.x * THREADS;
  for (size_t i = (size_t)blockIdx.x * THREADS + threadIdx.x; i < n; i += step) {
    const uint32_t v = __float_as_uint(a.data[i]);
    for (int q = 0; q < W; ++q)
      st_ll(static_cast<uint2*>(a.buf[q]) + ((size_t)par * W + a.rank) * stride + i, v, E);
  }
  for (size_t i = (size_t)blockIdx.x * THREADS + threadIdx.x; i < n; i += step) {
    float acc = 0.f;
    for (int q = 0; q < W; ++q)
      acc += __uint_as_float(wait_ll(static_cast<const uint2*>(a.buf[a.rank]) + ((size_t)par * W + q) * stride + i, E,
                                     budget, a.err, &give_up));
    a.data[i] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(a.grid_counter, 1u) + 1;
    if (done % gridDim.x == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch) = E;
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
  if (a.oneshot[0] != nullptr && a.rows <= FAR_SMALL_ROWS) {
    // Slices of whole warps (words per CTA a multiple of 32) keep every shuffle warp-uniform.
    if ((a.hidden / 2) % zs::coll::SMALL_CTAS != 0 || (a.hidden / 2) / zs::coll::SMALL_CTAS > zs::coll::THREADS * 4 ||
        ((a.hidden / 2) / zs::coll::SMALL_CTAS) % 32 != 0)
      return -1;
    for (int r = 0; r < a.world; ++r)
      if (a.oneshot[r] == nullptr) return -1;
    zs::coll::fused_allreduce_norm_small_kernel<<<FAR_SMALL_ROWS * zs::coll::SMALL_CTAS, zs::coll::THREADS, 0, stream>>>(
        a);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
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

extern "C" int zs_allreduce_sum_f32(const SumArArgs* args, cudaStream_t stream) {
  const SumArArgs& a = *args;
  if (a.world < 1 || a.world > 8 || a.rows < 0 || a.rows > a.max_rows || a.cols <= 0) return -1;
  for (int r = 0; r < a.world; ++r)
    if (a.buf[r] == nullptr) return -1;
  if (a.rows == 0) return 0;
  // A fixed grid keeps the completion counter a multiple of the grid across calls.
  zs::coll::allreduce_sum_f32_kernel<<<SUM_CTAS, zs::coll::THREADS, 0, stream>>>(a);
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

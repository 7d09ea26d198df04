// Expert-parallel MoE all-to-all over NVLink peer memory: dispatch and combine.
//
// Rank r owns routed experts [r*E/W, (r+1)*E/W).  Every rank allocates one symmetric
// block (cudaMalloc + CUDA IPC, layout in zs_kernels.h) and the kernels store straight
// into the peers' blocks; no staging copy, host memory or library collective sits on
// the data path.
//
// dispatch (one cooperative launch, G CTAs):
//   1. every (token, k) pair takes a slot in its expert's per-rank counter;
//   2. every rank publishes its per-expert counts to every rank (flag-in-data words
//      tagged with the call's epoch), so each rank knows the whole W x E count matrix;
//   3. every CTA derives the receive layout of every rank from the matrix: expert
//      segments in expert order, 128-row aligned (the grouped GEMM's tiles), and inside
//      a segment the sources in rank order;
//   4. one warp per token quantizes the bf16 row to MXFP8 once (16 columns per lane,
//      32-column e8m0 blocks) and stores the bytes, the scale atoms and a metadata word
//      into the segment of each top-k expert, on whichever rank owns it;
//   5. fence, grid barrier, one release flag per destination; the receiver waits for
//      every source and writes its grouped-GEMM metadata (counts, 128-row aligned
//      offsets, chunk prefix: the format of zs_moe_route) and marks padding rows.
//   Buffer reuse needs no extra handshake: a sender writes call E+1's rows only after it
//   has seen every rank's call E+1 counts, which a rank publishes only once its stream
//   has finished consuming call E (the grouped GEMMs and the combine run before the next
//   dispatch on every rank's stream).
//
// combine (one cooperative launch):
//   1. one warp per received row stores the expert output row (bf16) into its source's
//      return buffer at slot token * top_k + k;
//   2. fence, grid barrier, release flags; every CTA waits for every rank;
//   3. one warp per local token sums its top-k returned rows in k order with the routing
//      weights (+ residual) in fp32 and writes bf16.  The order is fixed, so the result
//      does not depend on arrival order.
//
// Every wait is bounded (timeout_ms): a missing peer records kErrPeerTimeout and the
// kernel returns.  Capacity overflow (more rows for some rank than recv_cap) is seen
// identically by every rank from the count matrix: all ranks record kErrBadShape, store
// nothing and hand the GEMM an empty work list.
//
// Reference parity: the reference serves experts tensor-parallel over host shared memory
// and has no all-to-all; this replaces the dispatch/combine of expert parallelism named
// for its DeepSeek configuration (worker/zstep_worker/models/deepseek_v41.py EP=8 path)
// and uses the routing format of its moe_align step (csrc/qwen35_ops_kernels.cu:26).
#include "peer.cuh"
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace ep {

using namespace peer;

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr uint32_t kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t* flags_of(const EpArgs& a, int r) {
  return reinterpret_cast<uint32_t*>(a.sym[r] + a.off_flags);
}
__device__ __forceinline__ uint2* counts_of(const EpArgs& a, int r) {
  return reinterpret_cast<uint2*>(a.sym[r] + a.off_counts);
}
__device__ __forceinline__ uint8_t* q_of(const EpArgs& a, int r) {
  return reinterpret_cast<uint8_t*>(a.sym[r] + a.off_q);
}
__device__ __forceinline__ uint8_t* sf_of(const EpArgs& a, int r) {
  return reinterpret_cast<uint8_t*>(a.sym[r] + a.off_sf);
}
__device__ __forceinline__ int2* meta_of(const EpArgs& a, int r) {
  return reinterpret_cast<int2*>(a.sym[r] + a.off_meta);
}
__device__ __forceinline__ __nv_bfloat16* comb_of(const EpArgs& a, int r) {
  return reinterpret_cast<__nv_bfloat16*>(a.sym[r] + a.off_comb);
}

// Grid barrier of a cooperative launch over a monotonic 64-bit counter: round n ends
// when the counter reaches n * G.  Bounded; on timeout it records kErrPeerTimeout.
__device__ __forceinline__ void grid_sync(unsigned long long* bar, unsigned long long G, uint64_t budget,
                                          int* err, volatile int* give_up) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long arrived = atomicAdd(bar, 1ull) + 1ull;
    const unsigned long long target = (arrived + G - 1) / G * G;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(bar) : "memory");
      if (v >= target) break;
      if ((i & 63) == 63) {
        if (globaltimer_ns() - t0 > budget) {
          report_error(err, kErrPeerTimeout);
          *give_up = 1;
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(THREADS) dispatch_kernel(const EpArgs a) {
  __shared__ int base_s[EP_MAX_EXPERTS];  // this rank's first row in each expert's segment (at its owner)
  __shared__ int tot_s[EP_MAX_EXPERTS];   // rows of each expert over all sources
  __shared__ int seg_s[EP_MAX_EXPERTS];   // segment base of each expert in its owner's buffer
  __shared__ int give_up, overflow;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = a.world, NE = a.num_experts, EL = NE / W, K = a.top_k, T = a.tokens, H = a.hidden;
  const unsigned long long G = gridDim.x;
  const uint32_t E = *reinterpret_cast<volatile uint32_t*>(a.epoch) + 1u;
  const uint64_t budget = limit_ns(a.timeout_ms);
  if (tid == 0) {
    give_up = 0;
    overflow = 0;
  }
  __syncthreads();

  // 1. slots in the per-expert counters of this rank
  for (int p = blockIdx.x * THREADS + tid; p < T * K; p += (int)G * THREADS) {
    const int e = a.topk_ids[p];
    a.pair_slot[p] = (e >= 0 && e < NE) ? atomicAdd(a.cnt + e, 1) : -1;
  }
  grid_sync(a.bar, G, budget, a.err, &give_up);

  // 2. this rank's count vector -> row `rank` of every rank's count matrix
  for (int d = blockIdx.x; d < W; d += (int)G) {
    uint2* dst = counts_of(a, d) + (size_t)a.rank * NE;
    for (int e = tid; e < NE; e += THREADS)
      st_ll(dst + e, (uint32_t)*reinterpret_cast<volatile int*>(a.cnt + e), E);
  }

  // 3. the whole matrix -> every rank's segment layout
  const uint2* cm = counts_of(a, a.rank);
  for (int e = tid; e < NE; e += THREADS) {
    int tot = 0, pre = 0;
    for (int s = 0; s < W; ++s) {
      const int c = (int)wait_ll(cm + (size_t)s * NE + e, E, budget, a.err, &give_up);
      tot += c;
      if (s < a.rank) pre += c;
    }
    tot_s[e] = tot;
    base_s[e] = pre;
  }
  __syncthreads();
  for (int d = warp; d < W; d += WARPS) {  // warp d: exclusive scan of d's aligned segments
    int run = 0;
    for (int e0 = d * EL; e0 < (d + 1) * EL; e0 += 32) {
      const int e = e0 + lane;
      const int v = e < (d + 1) * EL ? (tot_s[e] + 127) & ~127 : 0;
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += n;
      }
      if (e < (d + 1) * EL) seg_s[e] = run + inc - v;
      run += __shfl_sync(kFull, inc, 31);
    }
    if (lane == 0 && run > a.recv_cap) overflow = 1;
  }
  __syncthreads();
  const bool ovf = overflow != 0 || give_up != 0;  // overflow: identical on every rank
  for (int e = tid; e < NE; e += THREADS) base_s[e] += seg_s[e];
  __syncthreads();

  // 4. rows: one warp per token, quantized once, stored to each of its experts' owners
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a.x);
  for (int t = blockIdx.x * WARPS + warp; t < T; t += (int)G * WARPS) {
    int my_d = 0, my_row = -1;
    if (lane < K) {
      const int e = a.topk_ids[t * K + lane];
      const int slot = a.pair_slot[t * K + lane];
      if (slot >= 0) {
        if (ovf) {
          a.pair_slot[t * K + lane] = -1;  // the combine skips dropped pairs
        } else {
          my_d = e / EL;
          my_row = base_s[e] + slot;
          meta_of(a, my_d)[my_row] =
              make_int2((a.rank << 24) | (t * K + lane), __float_as_int(a.topk_w[t * K + lane]));
        }
      }
    }
    if (ovf) continue;
    const __nv_bfloat16* xr = x + (size_t)t * H;
    for (int c0 = 0; c0 < H; c0 += 512) {
      const int col = c0 + lane * 16;
      float f[16];
      unpack8(*reinterpret_cast<const uint4*>(xr + col), f);
      unpack8(*reinterpret_cast<const uint4*>(xr + col + 8), f + 8);
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(f[j]));
      amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));  // lanes 2i, 2i+1 share a 32-column block
      const uint8_t code = mx_scale_e8m0(amax);
      const float inv = mx_inv_scale(code);
      uint32_t w4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        w4[j] = uint32_t(f32_to_e4m3(f[4 * j] * inv)) | (uint32_t(f32_to_e4m3(f[4 * j + 1] * inv)) << 8) |
                (uint32_t(f32_to_e4m3(f[4 * j + 2] * inv)) << 16) |
                (uint32_t(f32_to_e4m3(f[4 * j + 3] * inv)) << 24);
      }
      const uint4 qv = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      // The four scale codes of a 128-column group (lanes g, g+2, g+4, g+6) are
      // contiguous bytes of the atom row: one 4-byte store.
      const int g = lane & ~7;
      const uint32_t sfw = uint32_t(__shfl_sync(kFull, (int)code, g)) |
                           (uint32_t(__shfl_sync(kFull, (int)code, g + 2)) << 8) |
                           (uint32_t(__shfl_sync(kFull, (int)code, g + 4)) << 16) |
                           (uint32_t(__shfl_sync(kFull, (int)code, g + 6)) << 24);
      for (int k = 0; k < K; ++k) {
        const int row = __shfl_sync(kFull, my_row, k);
        const int d = __shfl_sync(kFull, my_d, k);
        if (row < 0) continue;
        *reinterpret_cast<uint4*>(q_of(a, d) + (size_t)row * H + col) = qv;
        if ((lane & 7) == 0) {
          const size_t so = ((size_t)(row >> 7) * (H >> 7) + (col >> 7)) * 512 + sf_atom_offset(row & 127, 0);
          *reinterpret_cast<uint32_t*>(sf_of(a, d) + so) = sfw;
        }
      }
    }
  }

  // 5. publish, then (CTA 0) wait for every source and write the local GEMM metadata
  __threadfence_system();
  grid_sync(a.bar, G, budget, a.err, &give_up);
  if (blockIdx.x != 0) return;
  if (tid < W) st_release_sys(flags_of(a, tid) + a.rank, E);
  if (tid == 0) {
    for (int s = 0; s < W && !give_up; ++s) {
      if (!wait_flag_sys(flags_of(a, a.rank) + s, E, budget, nullptr)) {
        report_error(a.err, kErrPeerTimeout);
        give_up = 1;
      }
    }
    if (overflow) report_error(a.err, kErrBadShape);
  }
  __syncthreads();
  const int e_lo = a.rank * EL;
  if (warp == 0) {
    int run_c = 0;
    for (int e0 = 0; e0 < EL; e0 += 32) {
      const int e = e0 + lane;
      const int cnt = (e < EL && !ovf) ? tot_s[e_lo + e] : 0;
      const int ch = (cnt + a.chunk_rows - 1) / a.chunk_rows;
      int inc = ch;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += n;
      }
      if (e < EL) {
        a.group_count[e] = cnt;
        a.group_offset[e] = ovf ? 0 : seg_s[e_lo + e];
        a.chunk_prefix[e] = run_c + inc - ch;
      }
      run_c += __shfl_sync(kFull, inc, 31);
    }
    if (lane == 0) {
      a.chunk_prefix[EL] = run_c;
      const int last = e_lo + EL - 1;
      *a.recv_rows = ovf ? 0 : seg_s[last] + ((tot_s[last] + 127) & ~127);
    }
  }
  if (!ovf) {  // padding rows of the local segments carry no pair
    int2* meta = meta_of(a, a.rank);
    for (int e = warp; e < EL; e += WARPS) {
      const int lo = seg_s[e_lo + e] + tot_s[e_lo + e];
      const int hi = seg_s[e_lo + e] + ((tot_s[e_lo + e] + 127) & ~127);
      for (int r = lo + lane; r < hi; r += 32) meta[r] = make_int2(-1, 0);
    }
  }
  for (int e = tid; e < NE; e += THREADS) a.cnt[e] = 0;  // every CTA passed step 2's reads
  if (tid == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch) = E;
}

__global__ void __launch_bounds__(THREADS) combine_kernel(const EpArgs a) {
  __shared__ int give_up;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = a.world, NE = a.num_experts, K = a.top_k, T = a.tokens, H = a.hidden;
  const unsigned long long G = gridDim.x;
  const uint32_t E = *reinterpret_cast<volatile uint32_t*>(a.epoch + 1) + 1u;
  const uint64_t budget = limit_ns(a.timeout_ms);
  if (tid == 0) give_up = 0;
  __syncthreads();

  // 1. expert outputs back to their sources
  int R = *a.recv_rows;
  if (R > a.y_rows) {
    if (blockIdx.x == 0 && tid == 0) report_error(a.err, kErrBadShape);
    R = a.y_rows;  // rows past y are not sent; their tokens miss those terms
  }
  const int2* meta = meta_of(a, a.rank);
  const __nv_bfloat16* y = static_cast<const __nv_bfloat16*>(a.y);
  for (int i = blockIdx.x * WARPS + warp; i < R; i += (int)G * WARPS) {
    const int code = __ldcg(&meta[i].x);
    if (code < 0) continue;
    __nv_bfloat16* dst = comb_of(a, code >> 24) + (size_t)(code & 0xFFFFFF) * H;
    const __nv_bfloat16* src = y + (size_t)i * a.ldy;
    for (int c0 = lane * 8; c0 < H; c0 += 256 * 8) {  // 8 loads in flight, then 8 stores
      uint4 buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u * 256 < H) buf[u] = *reinterpret_cast<const uint4*>(src + c0 + u * 256);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u * 256 < H) *reinterpret_cast<uint4*>(dst + c0 + u * 256) = buf[u];
    }
  }
  __threadfence_system();
  grid_sync(a.bar, G, budget, a.err, &give_up);
  if (blockIdx.x == 0) {
    if (tid < W) st_release_sys(flags_of(a, tid) + 8 + a.rank, E);
    if (tid == 0) *reinterpret_cast<volatile uint32_t*>(a.epoch + 1) = E;  // all CTAs read it before the barrier
  }
  // 2. every rank's rows for this rank's tokens
  if (tid == 0) {
    for (int s = 0; s < W && !give_up; ++s) {
      if (!wait_flag_sys(flags_of(a, a.rank) + 8 + s, E, budget, nullptr)) {
        report_error(a.err, kErrPeerTimeout);
        give_up = 1;
      }
    }
  }
  __syncthreads();
  if (give_up) return;
  // 3. weighted sum in k order (+ residual)
  const __nv_bfloat16* comb = comb_of(a, a.rank);
  const __nv_bfloat16* res = static_cast<const __nv_bfloat16*>(a.residual);
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
  for (int t = blockIdx.x * WARPS + warp; t < T; t += (int)G * WARPS) {
    int my_ok = 0;
    float my_w = 0.f;
    if (lane < K) {
      const int e = a.topk_ids[t * K + lane];
      my_ok = (e >= 0 && e < NE && a.pair_slot[t * K + lane] >= 0) ? 1 : 0;
      my_w = a.topk_w[t * K + lane];
    }
    const unsigned okm = __ballot_sync(kFull, my_ok);  // bit k: pair k returned a row
    float wk[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) wk[k] = __shfl_sync(kFull, my_w, k);
    const __nv_bfloat16* crow = comb + (size_t)t * K * H;
    for (int c = lane * 8; c < H; c += 256) {
      // All top-k loads first (uncached: peers wrote them), then the sum in k order.
      uint4 v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (k < K && ((okm >> k) & 1u)) v[k] = __ldcv(reinterpret_cast<const uint4*>(crow + (size_t)k * H + c));
      float acc[8];
      if (res != nullptr) {
        unpack8(*reinterpret_cast<const uint4*>(res + (size_t)t * H + c), acc);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        if (k >= K || !((okm >> k) & 1u)) continue;
        float f[8];
        unpack8(v[k], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += wk[k] * f[j];
      }
      *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = pack8(acc);
    }
  }
}

int num_ctas() {
  static int n[16] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16) return 148;
  if (n[dev] == 0) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = sms > 0 ? sms : 148;
  }
  return n[dev];
}

int launch_coop(void (*kernel)(const EpArgs), const EpArgs& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_ctas());
  cfg.blockDim = dim3(THREADS);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a) == cudaSuccess ? 0 : -2;
}

bool valid(const EpArgs& a) {
  if (a.world < 1 || a.world > EP_MAX_WORLD || a.rank < 0 || a.rank >= a.world) return false;
  if (a.num_experts <= 0 || a.num_experts > EP_MAX_EXPERTS || a.num_experts % a.world != 0) return false;
  if (a.top_k <= 0 || a.top_k > 16 || a.hidden <= 0 || a.hidden % 512 != 0) return false;
  if (a.tokens < 0 || a.tokens > a.max_tokens || (long long)a.max_tokens * a.top_k >= (1 << 24)) return false;
  if (a.recv_cap <= 0 || a.recv_cap % 128 != 0 || (a.chunk_rows != 32 && a.chunk_rows != 128)) return false;
  for (int r = 0; r < a.world; ++r)
    if (a.sym[r] == nullptr) return false;
  return true;
}

}  // namespace ep
}  // namespace zs

extern "C" int zs_ep_dispatch(const EpArgs* args, cudaStream_t stream) {
  if (!zs::ep::valid(*args) || (args->x == nullptr && args->tokens > 0)) return -1;
  return zs::ep::launch_coop(zs::ep::dispatch_kernel, *args, stream);
}

extern "C" int zs_ep_combine(const EpArgs* args, cudaStream_t stream) {
  if (!zs::ep::valid(*args) || (args->y == nullptr && args->y_rows > 0) || (args->out == nullptr && args->tokens > 0))
    return -1;
  return zs::ep::launch_coop(zs::ep::combine_kernel, *args, stream);
}

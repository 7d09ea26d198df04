// MoE routing for the grouped MXFP8 expert GEMMs.
//
//   route_topk : one warp per token.  Softmax (Qwen), or sigmoid / sqrt(softplus) scores +
//                correction bias with grouped top-k (DeepSeek style) scoring, top-k with the
//                smallest-index tie break, optional renormalisation, then a slot in
//                the expert's segment via an atomic per-expert counter.  Experts
//                outside [expert_begin, expert_end) belong to other expert-parallel
//                ranks and are skipped; the shared expert (if any) is an extra local
//                group that every token visits with weight sigmoid(shared gate).
//   offsets    : one CTA; 128-row aligned segment offsets and the per-group prefix
//                of 128-token chunks that the GEMM's work list is built from.
//   scatter    : copies each routed token's MXFP8 row and its scale bytes into the
//                expert's segment and records (destination pair row, weight) for the
//                down-projection epilogue.
//
// Reference parity: router softmax-256/top-8/renorm + shared gate
// (worker/zstep_worker/kernels_sm120/qwen35_ops.py:1165-1222), moe_align_block_size
// (csrc/qwen35_ops_kernels.cu:26), sigmoid/sqrt-softplus routers
// (kernels_sm120/moe_router.py:31-110).
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace moe {

constexpr int kMaxExperts = 512;
constexpr int kMaxTopK = 16;

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffff, v, o);
    const int i2 = __shfl_xor_sync(0xffffffff, i, o);
    if (v2 > v || (v2 == v && i2 < i)) {
      v = v2;
      i = i2;
    }
  }
}

// Router logit (row, col), summing the router GEMM's split-K partials in order.
__device__ __forceinline__ float logit(const MoeRouteArgs& a, int row, int col) {
  const float* lg = a.logits + (size_t)row * a.ld_logits + col;
  float v = lg[0];
  for (int s = 1; s < a.logit_splits; ++s) v += lg[s * a.logit_split_stride];
  return v;
}

// One warp per row.  PER = experts per lane (lane owns experts lane + 32*j), a
// compile-time constant so scores, selection keys and the chosen top-k stay in registers.
template <int PER>
__global__ void route_topk_kernel(const MoeRouteArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.rows) return;
  const int E = a.num_experts;
  float score[PER];   // routing weight source
  float choice[PER];  // selection key
  {
    // Router logits (sum of the router GEMM's K partials, in order), loads issued together.
    const float* lg = a.logits + (size_t)row * a.ld_logits;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      score[j] = e < E ? lg[e] : -INFINITY;
    }
    for (int sp = 1; sp < a.logit_splits; ++sp) {
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int e = lane + 32 * j;
        if (e < E) score[j] += lg[(size_t)sp * a.logit_split_stride + e];
      }
    }
  }
  if (a.scoring == 0) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER; ++j) mx = fmaxf(mx, score[j]);
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      score[j] = (lane + 32 * j) < E ? __expf(score[j] - mx) : 0.f;
      sum += score[j];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      score[j] *= inv;
      choice[j] = (lane + 32 * j) < E ? score[j] : -INFINITY;
    }
  } else {
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      // sqrt(softplus(x)) with softplus = x above 20 (log1p(exp(x)) rounds to x there).
      const float x = score[j];
      score[j] = e >= E ? 0.f : a.scoring == 2 ? sqrtf(x > 20.f ? x : log1pf(__expf(x))) : sigmoidf_(x);
      choice[j] = e < E ? score[j] + (a.bias ? a.bias[e] : 0.f) : -INFINITY;
    }
    if (a.n_group > 1) {
      // Group score = sum of the two best choice scores in the group; keep the best
      // topk_group groups, mask the rest.
      const int gsize = E / a.n_group;
      __shared__ float gscore_s[8][64];
      float* gs = gscore_s[threadIdx.x >> 5];
      for (int g = 0; g < a.n_group; ++g) {
        float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
          const int e = lane + 32 * j;
          if (e >= g * gsize && e < (g + 1) * gsize) {
            const float c = choice[j];
            if (c > b1) { b2 = b1; b1 = c; } else if (c > b2) { b2 = c; }
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float o1 = __shfl_xor_sync(0xffffffff, b1, o);
          const float o2 = __shfl_xor_sync(0xffffffff, b2, o);
          const float n1 = fmaxf(b1, o1);
          const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
          b1 = n1;
          b2 = n2;
        }
        if (lane == 0) gs[g] = b1 + b2;
      }
      __syncwarp();
      // Select topk_group groups (ties -> lower group index).
      uint64_t keep = 0;
      for (int r = 0; r < a.topk_group; ++r) {
        int best = -1;
        float bv = -INFINITY;
        for (int g = 0; g < a.n_group; ++g)
          if (!((keep >> g) & 1) && (best < 0 || gs[g] > bv)) { best = g; bv = gs[g]; }
        keep |= 1ull << best;
      }
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int e = lane + 32 * j;
        if (e < E && !((keep >> (e / gsize)) & 1)) choice[j] = -INFINITY;
      }
      __syncwarp();
    }
  }
  // Top-k by choice key (ties -> smaller expert id); lane k keeps pick k.
  int my_id = 0;
  float my_w = 0.f, wsum = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) {
    if (k >= a.top_k) break;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && (choice[j] > bv || (choice[j] == bv && e < bi))) { bv = choice[j]; bi = e; }
    }
    warp_argmax(bv, bi);
    // Owner lane removes the winner and publishes its weight.
    float w = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (lane + 32 * j == bi) { w = score[j]; choice[j] = -INFINITY; }
    w = __shfl_sync(0xffffffff, w, bi & 31);
    if (lane == k) { my_id = bi; my_w = w; }
    wsum += w;
  }
  // Lanes 0..top_k-1 write their pick; the arrival order of the slot counters only
  // decides a pair's row inside its expert's segment.
  const int K1 = a.top_k + 1;
  if (lane < a.top_k) {
    float w = my_w;
    if (a.norm_topk) w = w / (wsum > 0.f ? wsum : 1.f);
    w *= a.routed_scale;
    a.topk_ids[row * a.top_k + lane] = my_id;
    a.topk_w[row * a.top_k + lane] = w;
    int slot = -1;
    if (my_id >= a.expert_begin && my_id < a.expert_end)
      slot = atomicAdd(a.group_count + (my_id - a.expert_begin), 1);
    a.pair_slot[row * K1 + lane] = slot;
  } else if (lane == a.top_k) {
    const int G_local = a.expert_end - a.expert_begin;
    a.pair_slot[row * K1 + a.top_k] = a.has_shared ? atomicAdd(a.group_count + G_local, 1) : -1;
  }
}

__global__ void offsets_kernel(const MoeRouteArgs a, int groups) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  // Single CTA of 1024 threads (one group each, groups <= 1024): exclusive scans of the
  // 128-aligned segment sizes and of the per-group chunk counts, warp scans + one
  // warp over the 32 warp totals.
  __shared__ int wsum_s[32], wsum_c[32];
  __shared__ int overflow;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int cr = a.chunk_rows;
  const int cnt = t < groups ? a.group_count[t] : 0;
  int s = (cnt + 127) & ~127;
  int c = (cnt + cr - 1) / cr;
  int is = s, ic = c;  // inclusive warp scans
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ns = __shfl_up_sync(0xffffffff, is, o);
    const int nc = __shfl_up_sync(0xffffffff, ic, o);
    if (lane >= o) { is += ns; ic += nc; }
  }
  if (lane == 31) { wsum_s[w] = is; wsum_c[w] = ic; }
  __syncthreads();
  if (w == 0) {
    int vs = wsum_s[lane], vc = wsum_c[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ns = __shfl_up_sync(0xffffffff, vs, o);
      const int nc = __shfl_up_sync(0xffffffff, vc, o);
      if (lane >= o) { vs += ns; vc += nc; }
    }
    wsum_s[lane] = vs;  // inclusive totals per warp
    wsum_c[lane] = vc;
  }
  __syncthreads();
  const int base_s = w > 0 ? wsum_s[w - 1] : 0, base_c = w > 0 ? wsum_c[w - 1] : 0;
  const int ex_s = base_s + is - s, ex_c = base_c + ic - c;
  const int total_s = wsum_s[31], total_c = wsum_c[31];
  if (t == 0) overflow = total_s > a.max_grouped_rows;
  __syncthreads();
  if (t < groups) {
    a.group_offset[t] = ex_s;
    // On overflow the GEMMs see no work rather than run past the buffer.
    a.chunk_prefix[t] = overflow ? 0 : ex_c;
  }
  if (t == 0) {
    a.chunk_prefix[groups] = overflow ? 0 : total_c;
    if (overflow) report_error(a.err, kErrBadShape);
  }
}

// One warp per (row, pair): copy hidden bytes + hidden/32 scale bytes.
__global__ void scatter_kernel(const MoeRouteArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int K1 = a.top_k + 1;
  const int pair = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (pair >= a.rows * K1) return;
  const int row = pair / K1, j = pair % K1;
  const int slot = a.pair_slot[pair];
  if (slot < 0) {
    if (a.pair_src != nullptr && lane == 0) a.pair_src[pair] = -1;
    return;
  }
  int g;
  float w;
  if (j < a.top_k) {
    g = a.topk_ids[row * a.top_k + j] - a.expert_begin;
    w = a.topk_w[row * a.top_k + j];
  } else {
    g = a.expert_end - a.expert_begin;
    w = a.shared_gate_col >= 0 ? sigmoidf_(logit(a, row, a.shared_gate_col)) : 1.f;
  }
  const int dst = a.group_offset[g] + slot;
  if (dst >= a.max_grouped_rows) {  // overflow (reported by offsets_kernel)
    if (a.pair_src != nullptr && lane == 0) a.pair_src[pair] = -1;
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(a.x_q + (size_t)row * a.hidden);
  uint4* dq = reinterpret_cast<uint4*>(a.xg_q + (size_t)dst * a.hidden);
  for (int c = lane; c < a.hidden / 16; c += 32) dq[c] = src[c];
  const int nkb = a.hidden / 32;
  for (int kb = lane; kb < nkb; kb += 32) {
    const size_t so = ((size_t)(row >> 7) * (a.hidden >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3);
    const size_t dso = ((size_t)(dst >> 7) * (a.hidden >> 7) + (kb >> 2)) * 512 + sf_atom_offset(dst & 127, kb & 3);
    a.xg_sf[dso] = a.x_sf[so];
  }
  if (lane == 0) {
    if (a.row_dst != nullptr) a.row_dst[dst] = row * K1 + j;
    if (a.row_scale != nullptr) a.row_scale[dst] = w;
    if (a.pair_src != nullptr) {
      a.pair_src[pair] = dst;
      a.pair_w[pair] = w;
    }
  }
}

}  // namespace moe
}  // namespace zs

extern "C" int zs_moe_route(const MoeRouteArgs* args, cudaStream_t stream) {
  const MoeRouteArgs& a = *args;
  if (a.num_experts > zs::moe::kMaxExperts || a.top_k > zs::moe::kMaxTopK || a.top_k <= 0) return -1;
  if (a.n_group > 64 || (a.n_group > 1 && a.num_experts % a.n_group != 0)) return -1;
  if (a.hidden % 128 != 0) return -1;
  if (a.chunk_rows != 32 && a.chunk_rows != 128) return -1;
  const int groups = (a.expert_end - a.expert_begin) + (a.has_shared ? 1 : 0);
  if (groups > 1024) return -1;
  if (cudaMemsetAsync(a.group_count, 0, sizeof(int) * groups, stream) != cudaSuccess) return -2;
  if (a.rows == 0) {
    zs_launch(zs::moe::offsets_kernel, 1, 1024, 0, stream, a, groups);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
  int wpb = 8;
  {
    const dim3 grid((a.rows + 1) / 2), block(64);  // 2 rows per block: more SMs busy
    if (a.num_experts <= 64) zs_launch(zs::moe::route_topk_kernel<2>, grid, block, 0, stream, a);
    else if (a.num_experts <= 128) zs_launch(zs::moe::route_topk_kernel<4>, grid, block, 0, stream, a);
    else if (a.num_experts <= 256) zs_launch(zs::moe::route_topk_kernel<8>, grid, block, 0, stream, a);
    else zs_launch(zs::moe::route_topk_kernel<16>, grid, block, 0, stream, a);
  }
  zs_launch(zs::moe::offsets_kernel, 1, 1024, 0, stream, a, groups);
  const int pairs = a.rows * (a.top_k + 1);
  zs_launch(zs::moe::scatter_kernel, (pairs + wpb - 1) / wpb, wpb * 32, 0, stream, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

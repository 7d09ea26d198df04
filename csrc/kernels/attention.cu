// Gated GQA attention over a paged KV cache (Qwen3.5 full-attention layers).
//
// KV cache layout: [pages][kv_heads][16 tokens x 256 dims] bf16 blocks of 8 KiB, stored
// pre-swizzled for the tensor cores: a block holds two halves of 8 tokens, each half four
// 64-dim chunks of 8 rows x 128 B, and the 16-byte pieces of token row r sit at piece
// index ^ (r % 8) (see swz()).  One cp.async.bulk copies a block into shared memory where
// it is directly a K-major operand (8-row groups 4 KiB apart) or, for V, an MN-major one.
//
//  * prologue: per row, zero-centered RMSNorm of every q and k head ((1 + w) scale),
//    partial rotary embedding (rotate-half over the first `rotary_dim` dims, cos/sin
//    rounded to bf16 as a bf16 rotary cache would be), sigmoid-gate passthrough, and
//    the K/V write into the row's page slot.
//  * split-KV decode: one CTA per (row, kv head, split), one warp per query head of the
//    GQA group.  Thread 0 streams the split's pages (K and V blocks) through a 4-deep
//    shared-memory ring with cp.async.bulk + mbarriers; each warp splits into 4 lane
//    groups that take one token each (8 lanes x 32 dims, bank-conflict-free 16-byte
//    pieces), with an online softmax per lane group.  Partials (o, m, l) go to scratch
//    and a combine kernel merges the splits, applies the sigmoid gate and emits bf16
//    and/or MXFP8 for the o_proj GEMM.
//  * varlen prefill reuses the same kernels with each query row's causal context length
//    (position + 1): K/V of the whole chunk are written first, then every query row
//    attends over its own prefix.
//
// Reference parity: worker/zstep_worker/kernels_sm120/qwen35_ops.py:187-560 (attention
// prologue, split-K(16) paged GQA decode + gated reduce, varlen gated prefill).
#include <cstdio>
#include <mutex>

#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace attn {

constexpr int D = 256;       // head_dim supported by these kernels
constexpr int PAGE = 16;     // tokens per page
constexpr int RING = 4;      // staged pages per CTA
constexpr int BLOCK_BYTES = PAGE * D * 2;  // one (page, kv head) block: 8 KiB

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Element offset of the (page, kv head) block.
__device__ __forceinline__ size_t kv_offset(const AttnArgs& a, int page, int kvh) {
  return ((size_t)page * a.num_kv_heads + kvh) * PAGE * D;
}

// Element offset of (token row r, dims d..d+7) inside a block (d a multiple of 8).
__device__ __forceinline__ int swz(int r, int d) {
  return (r >> 3) * 2048 + (d >> 6) * 512 + (r & 7) * 64 + ((((d & 63) >> 3) ^ (r & 7)) << 3);
}

// One CTA per row; one warp per head (q heads then k heads then v heads); lane owns 8 dims.
__global__ void prologue_kernel(const AttnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nh = a.num_q_heads + a.num_kv_heads;
  const int pos = a.positions[row];
  const int half = a.rotary_dim / 2;
  const __nv_bfloat16* qkv = static_cast<const __nv_bfloat16*>(a.qkv) + (size_t)row * a.ld_qkv;
  const int slot = a.slots[row];
  const int page = a.page_table[(size_t)slot * a.max_pages + pos / a.page_size];
  for (int h = warp; h < nh + a.num_kv_heads; h += blockDim.x >> 5) {
    if (h >= nh) {
      // V head: straight copy into the cache.
      const int kvh = h - nh;
      const uint4* src = reinterpret_cast<const uint4*>(qkv + a.num_q_heads * 2 * D + a.num_kv_heads * D + kvh * D);
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.v_cache) + kv_offset(a, page, kvh) +
                                swz(pos % a.page_size, lane * 8)) =
          src[lane];
      continue;
    }
    const bool is_q = h < a.num_q_heads;
    const __nv_bfloat16* src = is_q ? qkv + h * 2 * D : qkv + a.num_q_heads * 2 * D + (h - a.num_q_heads) * D;
    const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(is_q ? a.q_norm_w : a.k_norm_w);
    float x[8];
    {
      uint4 u = reinterpret_cast<const uint4*>(src)[lane];
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(hh[j]);
        x[2 * j] = f.x;
        x[2 * j + 1] = f.y;
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / D + a.eps);
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = bfr(x[j] * rstd * (1.f + __bfloat162float(w[lane * 8 + j])));
    // Partial rope: dims [0, half) pair with [half, 2*half).  Lanes holding dims < half
    // fetch their partner from lane + half/8 and vice versa.
    const int d0 = lane * 8;
    const int partner_off = half / 8;
    float other[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float up = __shfl_down_sync(0xffffffff, y[j], partner_off);
      const float dn = __shfl_up_sync(0xffffffff, y[j], partner_off);
      other[j] = d0 < half ? up : dn;
    }
    if (d0 < 2 * half) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = d0 + j;
        const int i = d < half ? d : d - half;
        const float inv_freq = powf(a.rope_theta, -2.0f * i / a.rotary_dim);
        float sn, cs;
        sincosf((float)pos * inv_freq, &sn, &cs);
        cs = bfr(cs);
        sn = bfr(sn);
        y[j] = d < half ? bfr(y[j] * cs - other[j] * sn) : bfr(y[j] * cs + other[j] * sn);
      }
    }
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 b = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
      packed[j] = *reinterpret_cast<uint32_t*>(&b);
    }
    const uint4 pv = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    if (is_q) {
      __nv_bfloat16* qo = static_cast<__nv_bfloat16*>(a.q_out) + ((size_t)row * a.num_q_heads + h) * D;
      reinterpret_cast<uint4*>(qo)[lane] = pv;
      __nv_bfloat16* go = static_cast<__nv_bfloat16*>(a.gate_out) + ((size_t)row * a.num_q_heads + h) * D;
      reinterpret_cast<uint4*>(go)[lane] = reinterpret_cast<const uint4*>(src + D)[lane];
    } else {
      const int kvh = h - a.num_q_heads;
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.k_cache) + kv_offset(a, page, kvh) +
                                swz(pos % a.page_size, lane * 8)) =
          pv;
    }
  }
}

// Partial record per (row, q head, split): o[256] (unnormalised), m, l, 2 pad floats.
constexpr int PREC = D + 4;  // padded to keep each record 16-byte aligned

struct DecSmem {
  __nv_bfloat16 k[RING][PAGE * D];
  __nv_bfloat16 v[RING][PAGE * D];
  uint64_t full[RING];
  uint64_t empty[RING];
  int abort_flag;
};

// Lane li of a lane group owns dims {c*64 + li*8 + 0..7 : c = 0..3}: a quarter-warp's
// 16-byte accesses then cover 128 contiguous bytes (no bank conflicts).
__device__ __forceinline__ void load_row_piece(const __nv_bfloat16* row, int li, float (&f)[32]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + c * 64 + li * 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&u)[j]);
      f[c * 8 + 2 * j] = v.x;
      f[c * 8 + 2 * j + 1] = v.y;
    }
  }
}

// The same pieces of token row t of a swizzled (page, kv head) block.
__device__ __forceinline__ void load_block_row_piece(const __nv_bfloat16* blk, int t, int li, float (&f)[32]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(blk + swz(t, c * 64 + li * 8));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 v = __bfloat1622float2(h[j]);
      f[c * 8 + 2 * j] = v.x;
      f[c * 8 + 2 * j + 1] = v.y;
    }
  }
}

__global__ void __launch_bounds__(256) decode_partial_kernel(const AttnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t dec_smem_raw[];
  DecSmem& s = *reinterpret_cast<DecSmem*>((reinterpret_cast<uintptr_t>(dec_smem_raw) + 127) & ~uintptr_t(127));
  const int row = blockIdx.x;
  const int kvh = blockIdx.y;
  const int split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int group = a.num_q_heads / a.num_kv_heads;
  const int qh = kvh * group + warp;
  const int grp = lane >> 3, li = lane & 7;
  const int ctx = a.seq_lens[row];
  const int slot = a.slots[row];
  // Pages of this split.
  const int pages = (ctx + PAGE - 1) / PAGE;
  const int pps = (pages + a.num_splits - 1) / a.num_splits;
  const int p0 = split * pps;
  const int p1 = min(pages, p0 + pps);
  const int npg = max(0, p1 - p0);
  const int* pt = a.page_table + (size_t)slot * a.max_pages;
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(a.k_cache);
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(a.v_cache);
  volatile int* abort_flag = &s.abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RING; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], nwarps);
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int pi) {
    const int st = pi % RING;
    const int page = __ldg(pt + p0 + pi);
    mbar_expect_tx(&s.full[st], 2 * BLOCK_BYTES);
    bulk_load(s.k[st], kc + kv_offset(a, page, kvh), BLOCK_BYTES, &s.full[st]);
    bulk_load(s.v[st], vc + kv_offset(a, page, kvh), BLOCK_BYTES, &s.full[st]);
  };
  if (threadIdx.x == 0)
    for (int pi = 0; pi < min(RING, npg); ++pi) issue(pi);

  const float qscale = a.sm_scale * 1.4426950408889634f;  // exp2 domain
  float q[32];
  load_row_piece(static_cast<const __nv_bfloat16*>(a.q_out) + ((size_t)row * a.num_q_heads + qh) * D, li, q);
#pragma unroll
  for (int j = 0; j < 32; ++j) q[j] *= qscale;
  float o[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j] = 0.f;
  float m = -INFINITY, l = 0.f;

  int pi = 0;
  for (; pi < npg; ++pi) {
    const int st = pi % RING;
    bool ok = true;
    for (uint32_t it = 0; !mbar_try_wait(&s.full[st], (pi / RING) & 1); ++it) {
      if (*abort_flag || it > kMbarSpinLimit) { ok = false; break; }
    }
    if (!__all_sync(0xffffffff, ok)) {
      report_error(a.err, kErrMbarTimeout);
      *abort_flag = 1;
      break;
    }
    const int tok0 = (p0 + pi) * PAGE;
#pragma unroll 1
    for (int t = grp; t < PAGE; t += 4) {
      const bool valid = tok0 + t < ctx;
      float kf[32];
      load_block_row_piece(s.k[st], t, li, kf);
      float sc = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) sc += q[j] * kf[j];
      sc += __shfl_xor_sync(0xffffffff, sc, 1);
      sc += __shfl_xor_sync(0xffffffff, sc, 2);
      sc += __shfl_xor_sync(0xffffffff, sc, 4);
      if (!valid) continue;
      float vf[32];
      load_block_row_piece(s.v[st], t, li, vf);
      if (sc > m) {
        const float r = exp2f(m - sc);
        l *= r;
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] *= r;
        m = sc;
      }
      const float p = exp2f(sc - m);
      l += p;
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] += p * vf[j];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.empty[st]);
    // Refill this stage with page pi + RING once every warp is done with it.
    if (threadIdx.x == 0 && pi + RING < npg) {
      if (!mbar_wait(&s.empty[st], (pi / RING) & 1, a.err)) {
        *abort_flag = 1;
      } else {
        issue(pi + RING);
      }
    }
  }
  // Drain (abort path): wait for copies that were issued but not consumed.
  if (threadIdx.x == 0) {
    const int issued = min(npg, pi + RING);
    for (int j = pi; j < issued; ++j) mbar_wait(&s.full[j % RING], (j / RING) & 1, nullptr);
  }
  // Merge the 4 lane groups (xor 8, xor 16 pair groups with equal li).
#pragma unroll
  for (int off = 8; off <= 16; off <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffff, m, off);
    const float l2 = __shfl_xor_sync(0xffffffff, l, off);
    const float mn = fmaxf(m, m2);
    const float s1 = (m == -INFINITY) ? 0.f : exp2f(m - mn);
    const float s2 = (m2 == -INFINITY) ? 0.f : exp2f(m2 - mn);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float o2 = __shfl_xor_sync(0xffffffff, o[j], off);
      o[j] = o[j] * s1 + o2 * s2;
    }
    l = l * s1 + l2 * s2;
    m = mn;
  }
  if (grp == 0) {
    float* rec = a.partial + (((size_t)row * a.num_q_heads + qh) * a.num_splits + split) * PREC;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float4* dst = reinterpret_cast<float4*>(rec + c * 64 + li * 8);
      dst[0] = make_float4(o[c * 8], o[c * 8 + 1], o[c * 8 + 2], o[c * 8 + 3]);
      dst[1] = make_float4(o[c * 8 + 4], o[c * 8 + 5], o[c * 8 + 6], o[c * 8 + 7]);
    }
    if (li == 0) {
      rec[D] = m;
      rec[D + 1] = l;
    }
  }
}

// ---------------------------------------------------------------------------------
// Tensor-core split-KV decode (tcgen05).  One CTA of 4 warps per (row, kv head, split);
// the split's keys go through 128-key tiles (8 pages):
//   * One cp.async.bulk per page copies each pre-swizzled (page, kv head) block of K and V
//     into the tile image: page j at 8 KiB * j, so for every 64-dim chunk the tile's
//     128 key rows form 16 groups of 8 rows, 4 KiB apart (the operand's SBO).
//   * S^T = K Q^T: one thread issues 16 tcgen05.mma (kind::f16 bf16, M = 128 keys,
//     N = 16 query-head slots of the GQA group, K = 16 dims each) into TMEM columns 0-15.
//   * Online softmax in the exp2 domain: thread t owns key t (TMEM lane t); per-head
//     maxima and sums reduce through shared memory; P = exp2(S - m) is stored bf16 as
//     the [16 heads x 128 keys] K-major operand of the second product, and O is rescaled
//     in TMEM (tcgen05.ld / st) by exp2(m_old - m_new).
//   * O^T += V^T P^T: the V tile image read as an MN-major operand (M = 128 head dims per
//     MMA: 64-dim chunks LBO = 1 KiB apart, 8-key groups SBO = 4 KiB apart), N = 16,
//     K = 16 keys (one page) per MMA, accumulated in TMEM columns 16-47.
// K is reloaded as soon as S is in TMEM; V images are double-buffered and requested two
// tiles ahead, so both copies overlap the dependent chain of a tile.  Output
// records (o, m, l) have the layout of the SIMT kernel, so the same combine kernel runs.
constexpr int TC_KEYS = 128;
constexpr int TC_PAGES = TC_KEYS / PAGE;
constexpr int TC_N = 16;
constexpr int TC_NCHUNK = D / 64;
constexpr int TC_TILE_BYTES = TC_PAGES * BLOCK_BYTES;
constexpr int TC_THREADS = 128;

struct TcSmem {
  uint8_t k[TC_TILE_BYTES];           // K tile image (reloaded as soon as S is computed)
  uint8_t v[2][TC_TILE_BYTES];        // double-buffered V tile images (prefetched two tiles ahead)
  uint8_t q[TC_NCHUNK][TC_N * 128];   // Q: [16 slots][256] K-major, slots >= group are zero
  uint8_t p[2][TC_N * 128];           // P: [16 slots][128 keys] K-major, 2 chunks of 64 keys
  float red_max[4][TC_N];
  float red_sum[4][TC_N];
  float m[TC_N], l[TC_N], r[TC_N];
  uint64_t kfull, vfull[2], mma1, mma2;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(TC_THREADS, 1)
decode_partial_tc_kernel(const AttnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  TcSmem& s = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.num_q_heads / a.num_kv_heads;
  const int ctx = a.seq_lens[row];
  const int pages = (ctx + PAGE - 1) / PAGE;
  const int pps = (pages + a.num_splits - 1) / a.num_splits;
  const int p0 = split * pps;
  const int p1 = min(pages, p0 + pps);
  const int npg = max(0, p1 - p0);
  const int ntiles = (npg + TC_PAGES - 1) / TC_PAGES;
  const int tok_end = min(ctx, p1 * PAGE);
  const int* pt = a.page_table + (size_t)a.slots[row] * a.max_pages;
  const float qscale = a.sm_scale * 1.4426950408889634f;  // exp2 domain

  if (warp == 0) {
    tmem_alloc(&s.tmem_base, 64);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.kfull, 1);
    mbar_init(&s.vfull[0], 1);
    mbar_init(&s.vfull[1], 1);
    mbar_init(&s.mma1, 1);
    mbar_init(&s.mma2, 1);
    fence_barrier_init();
  }
  if (tid < TC_N) {
    s.m[tid] = -INFINITY;
    s.l[tid] = 0.f;
  }
  // Q slots of this kv head's GQA group (rows >= G stay zero).
  const __nv_bfloat16* qsrc = static_cast<const __nv_bfloat16*>(a.q_out) + ((size_t)row * a.num_q_heads + kvh * G) * D;
  for (int i = tid; i < TC_N * 32; i += TC_THREADS) {
    const int h = i >> 5, pc = i & 31, c = pc >> 3, piece = pc & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < G) v = *reinterpret_cast<const uint4*>(qsrc + (size_t)h * D + pc * 8);
    *reinterpret_cast<uint4*>(s.q[c] + h * 128 + ((piece ^ (h & 7)) << 4)) = v;
  }
  fence_proxy_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t t_s = tmem, t_o = tmem + 16;

  // Producer state (thread 0 only): loads issued but not yet observed, per barrier.
  int k_pend = 0, v_pend[2] = {0, 0};
  int k_uses = 0, v_uses[2] = {0, 0};
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(a.k_cache);
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(a.v_cache);
  // The tile's page ids are loaded together (independent loads, one latency), then its
  // page copies are issued back to back.
  auto issue = [&](const __nv_bfloat16* cache, uint8_t* dst, uint64_t* bar, int tile) {
    const int pg0 = p0 + tile * TC_PAGES;
    const int n = min(TC_PAGES, p1 - pg0);
    int page[TC_PAGES];
#pragma unroll
    for (int j = 0; j < TC_PAGES; ++j) page[j] = j < n ? __ldg(pt + pg0 + j) : 0;
    mbar_expect_tx(bar, n * BLOCK_BYTES);
#pragma unroll
    for (int j = 0; j < TC_PAGES; ++j)
      if (j < n) bulk_load(dst + j * BLOCK_BYTES, cache + kv_offset(a, page[j], kvh), BLOCK_BYTES, bar);
  };
  if (tid == 0 && ntiles > 0) {
    issue(kc, s.k, &s.kfull, 0);
    k_pend = 1;
    for (int j = 0; j < 2 && j < ntiles; ++j) {
      issue(vc, s.v[j], &s.vfull[j], j);
      v_pend[j] = 1;
    }
  }
  bool ok = true;
  for (int t = 0; t < ntiles; ++t) {
    const int vb = t & 1;
    const int pg0 = p0 + t * TC_PAGES;
    const int n = min(TC_PAGES, p1 - pg0);
    if (n < TC_PAGES) {
      // Last, partial tile: zero the absent pages in both images (no copy targets them),
      // so the products see finite values there.
      for (int i = n * (BLOCK_BYTES / 16) + tid; i < TC_PAGES * (BLOCK_BYTES / 16); i += TC_THREADS) {
        reinterpret_cast<uint4*>(s.k)[i] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(s.v[vb])[i] = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_shared();
    }
    ok = mbar_wait(&s.kfull, (uint32_t)(k_uses & 1), a.err);
    if (!__syncthreads_and(ok)) break;
    if (tid == 0) {
      k_pend = 0;
      tc_fence_after();
      const uint32_t idesc = make_idesc_bf16(TC_KEYS, TC_N, 0, 0);
#pragma unroll
      for (int c = 0; c < TC_NCHUNK; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ad = make_smem_desc(smem_u32(s.k + c * 1024) + k * 32, 16, 4096, 2);
          const uint64_t bd = make_smem_desc(smem_u32(s.q[c]) + k * 32, 16, 1024, 2);
          mma_bf16(t_s, ad, bd, idesc, (c | k) ? 1u : 0u);
        }
      tc_commit(&s.mma1);
    }
    ++k_uses;
    ok = mbar_wait(&s.mma1, (uint32_t)(t & 1), a.err);
    if (!__syncthreads_and(ok)) break;
    tc_fence_after();
    // S is in TMEM: the K image is free, so the next tile's K copy overlaps the rest of
    // this tile (softmax, rescale, second product).
    if (tid == 0 && t + 1 < ntiles) {
      issue(kc, s.k, &s.kfull, t + 1);
      k_pend = 1;
    }
    // ---- online softmax: thread tid owns key tid of the tile
    uint32_t sr[16];
    tmem_ld_32x32b_x16(t_s + lane_off, sr);
    tmem_ld_wait();
    const int tok = pg0 * PAGE + tid;
    const bool valid = tok < tok_end;
    float sv[TC_N];
#pragma unroll
    for (int h = 0; h < TC_N; ++h) sv[h] = (valid && h < G) ? __uint_as_float(sr[h]) * qscale : -INFINITY;
#pragma unroll
    for (int h = 0; h < TC_N; ++h) {
      const float v = warp_max(sv[h]);
      if (lane == 0) s.red_max[warp][h] = v;
    }
    __syncthreads();
    float mnew[TC_N];
#pragma unroll
    for (int h = 0; h < TC_N; ++h)
      mnew[h] = fmaxf(fmaxf(s.m[h], fmaxf(s.red_max[0][h], s.red_max[1][h])), fmaxf(s.red_max[2][h], s.red_max[3][h]));
    {
      const int chunk = tid >> 6, within = tid & 63, piece = within >> 3, sub = (within & 7) * 2;
#pragma unroll
      for (int h = 0; h < TC_N; ++h) {
        const float pv = sv[h] == -INFINITY ? 0.f : exp2f(sv[h] - mnew[h]);
        const __nv_bfloat16 pb = __float2bfloat16_rn(pv);
        *reinterpret_cast<__nv_bfloat16*>(s.p[chunk] + h * 128 + ((piece ^ (h & 7)) << 4) + sub) = pb;
        const float sum = warp_sum(__bfloat162float(pb));
        if (lane == 0) s.red_sum[warp][h] = sum;
      }
    }
    fence_proxy_async_shared();
    __syncthreads();
    if (tid < TC_N) {
      const int h = tid;
      const float mo = s.m[h];
      const float rr = mo == -INFINITY ? 0.f : exp2f(mo - mnew[h]);
      s.l[h] = s.l[h] * rr + (s.red_sum[0][h] + s.red_sum[1][h] + s.red_sum[2][h] + s.red_sum[3][h]);
      s.m[h] = mnew[h];
      s.r[h] = rr;
    }
    __syncthreads();
    if (t > 0) {  // rescale the running O^T (TMEM lane = head dim, column = head slot)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t o[16];
        tmem_ld_32x32b_x16(t_o + mt * 16 + lane_off, o);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 16; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * s.r[h]);
        tmem_st_32x32b_x16(t_o + mt * 16 + lane_off, o);
      }
      tmem_st_wait();
    }
    ok = mbar_wait(&s.vfull[vb], (uint32_t)(v_uses[vb] & 1), a.err);
    if (ok && !valid && tok < (pg0 + n) * PAGE) {
      // Cache rows past the context inside a loaded page: zero them (P is 0 there).
      const int r = tid & 15;
      uint8_t* blk = s.v[vb] + (tid >> 4) * BLOCK_BYTES + (r >> 3) * 4096 + (r & 7) * 128;
#pragma unroll
      for (int c = 0; c < TC_NCHUNK; ++c) {
        uint4* rowp = reinterpret_cast<uint4*>(blk + c * 1024);
#pragma unroll
        for (int j = 0; j < 8; ++j) rowp[j] = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_shared();
    }
    tc_fence_before();
    if (!__syncthreads_and(ok)) break;
    if (tid == 0) {
      v_pend[vb] = 0;
      tc_fence_after();
      const uint32_t idesc2 = make_idesc_bf16(128, TC_N, 1, 0);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t ad = make_smem_desc(smem_u32(s.v[vb] + 2 * mt * 1024) + ks * BLOCK_BYTES, 1024, 4096, 2);
          const uint64_t bd = make_smem_desc(smem_u32(s.p[ks >> 2]) + (ks & 3) * 32, 16, 1024, 2);
          mma_bf16(t_o + mt * 16, ad, bd, idesc2, (t > 0 || ks > 0) ? 1u : 0u);
        }
      tc_commit(&s.mma2);
    }
    ++v_uses[vb];
    ok = mbar_wait(&s.mma2, (uint32_t)(t & 1), a.err);
    if (!__syncthreads_and(ok)) break;
    tc_fence_after();
    if (tid == 0 && t + 2 < ntiles) {  // this V image is free: the tile after next
      issue(vc, s.v[vb], &s.vfull[vb], t + 2);
      v_pend[vb] = 1;
    }
  }
  if (ok) {
    const int h_lim = G < TC_N ? G : TC_N;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      uint32_t o[16];
      if (ntiles > 0) {
        tmem_ld_32x32b_x16(t_o + mt * 16 + lane_off, o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) o[h] = 0u;
      }
      const int dim = mt * 128 + tid;
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        if (h >= h_lim) break;
        a.partial[(((size_t)row * a.num_q_heads + kvh * G + h) * a.num_splits + split) * PREC + dim] =
            __uint_as_float(o[h]);
      }
    }
    if (tid < h_lim) {
      float* rec = a.partial + (((size_t)row * a.num_q_heads + kvh * G + tid) * a.num_splits + split) * PREC;
      rec[D] = s.m[tid];
      rec[D + 1] = s.l[tid];
    }
  } else {
    // Abort (the error word is set): still write an empty record (m = -inf, l = 0) for each
    // head of this split, so the combine kernel skips the split instead of reading whatever
    // an earlier call left in the scratch buffer.
    const int h_lim = G < TC_N ? G : TC_N;
    if (tid < h_lim) {
      float* rec = a.partial + (((size_t)row * a.num_q_heads + kvh * G + tid) * a.num_splits + split) * PREC;
      rec[D] = -INFINITY;
      rec[D + 1] = 0.f;
    }
    // Let every copy still in flight land before the CTA releases shared memory.
    if (tid == 0) {
      if (k_pend) mbar_wait(&s.kfull, (uint32_t)(k_uses & 1), nullptr);
      for (int b = 0; b < 2; ++b)
        if (v_pend[b]) mbar_wait(&s.vfull[b], (uint32_t)(v_uses[b] & 1), nullptr);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------------------------
// Tensor-core attention over query rows grouped by sequence (varlen prefill, speculative
// verify: seq_start given).  A work item is (query rows, kv head, split): up to NS / G
// consecutive rows of one sequence (NS = 32 query slots = row x head of the GQA group:
// 4 rows at G = 8, 16 at G = 2), so every K/V tile it loads serves all of them instead of
// one row, each slot masked by its own causal length.  Per 128-key tile the steps are
// those of the decode kernel above (page-image bulk copies, S^T = K Q^T with N = NS,
// online softmax with the TMEM rescale, O^T += V^T P^T), with these differences:
//   * each CTA walks items idx = blockIdx.x + j * gridDim.x, its copies running ahead over
//     its whole tile stream (K one tile, V two tiles) across item boundaries; the launch
//     covers every item with its own CTA (an upper bound on the item count), so a CTA
//     walks more than one item only when given a smaller grid;
//   * a tile's page ids are read together, then its page copies issued back to back;
//   * the item list is built in the CTA from seq_start: a scan of each sequence's row
//     chunks into shared memory, then a binary search per item.
// Records (o, m, l) per (row, head, split) feed the same combine kernel.
constexpr int TC_NMR = 32;         // query slots of a work item
constexpr int TC_MAX_SEQS = 1024;  // sequences whose chunk prefix fits in shared memory

template <int NS>
struct TcRowsSmem {
  uint8_t k[TC_TILE_BYTES];           // K tile image (reloaded as soon as S is computed)
  uint8_t v[2][TC_TILE_BYTES];        // double-buffered V tile images (prefetched two tiles ahead)
  uint8_t q[TC_NCHUNK][NS * 128];     // Q: [NS slots][256] K-major, unused slots are zero
  uint8_t p[2][NS * 128];             // P: [NS slots][128 keys] K-major, 2 chunks of 64 keys
  float red_max[4][NS];
  float red_sum[4][NS];
  float m[NS], l[NS], r[NS];
  int len[NS];                        // causal length of each slot's row (0: unused slot)
  int cpre[TC_MAX_SEQS + 1];          // items (row chunks) before each sequence
  int tsum[TC_THREADS + 1];
  uint64_t kfull, vfull[2], mma1, mma2;
  uint32_t tmem_base;
};

// One work item: query rows [r0, r0 + nr) of one sequence, a kv head and a split, whose
// keys are the pages [p0, p1) (the split's share of the longest row's context).
struct TcItem {
  int r0, nr, kvh, split, p0, p1, ntiles, tok_end;
  const int* pt;
};

// rpi = query rows per item; cpre = row-chunk prefix over the sequences.
__device__ __forceinline__ bool tc_item(const AttnArgs& a, int idx, int rpi, const int* cpre, TcItem& it) {
  if (idx >= cpre[a.num_seqs] * a.num_kv_heads * a.num_splits) return false;
  it.split = idx % a.num_splits;
  const int rk = idx / a.num_splits;
  it.kvh = rk % a.num_kv_heads;
  const int chunk = rk / a.num_kv_heads;
  int lo = 0, hi = a.num_seqs;  // largest sequence with cpre[seq] <= chunk
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cpre[mid] <= chunk) lo = mid; else hi = mid;
  }
  it.r0 = a.seq_start[lo] + (chunk - cpre[lo]) * rpi;
  it.nr = min(rpi, a.seq_start[lo + 1] - it.r0);
  int ctx = 0;
  for (int i = 0; i < it.nr; ++i) ctx = max(ctx, a.seq_lens[it.r0 + i]);
  const int pages = (ctx + PAGE - 1) / PAGE;
  const int pps = (pages + a.num_splits - 1) / a.num_splits;
  it.p0 = it.split * pps;
  it.p1 = min(pages, it.p0 + pps);
  it.ntiles = (max(0, it.p1 - it.p0) + TC_PAGES - 1) / TC_PAGES;
  it.tok_end = min(ctx, it.p1 * PAGE);
  it.pt = a.page_table + (size_t)a.slots[it.r0] * a.max_pages;
  return true;
}

// Copy-side position in the CTA's tile stream (thread 0 only): item j, tile t.
struct TcCursor {
  int j, t;
  bool valid;
  TcItem it;
};

__device__ __forceinline__ void tc_settle(const AttnArgs& a, int rpi, const int* cpre, TcCursor& c) {
  while (c.valid && c.t >= c.it.ntiles) {  // skip items without keys
    ++c.j;
    c.t = 0;
    c.valid = tc_item(a, blockIdx.x + c.j * gridDim.x, rpi, cpre, c.it);
  }
}

__device__ __forceinline__ void tc_start(const AttnArgs& a, int rpi, const int* cpre, TcCursor& c) {
  c.j = 0;
  c.t = 0;
  c.valid = tc_item(a, blockIdx.x, rpi, cpre, c.it);
  tc_settle(a, rpi, cpre, c);
}

__device__ __forceinline__ void tc_advance(const AttnArgs& a, int rpi, const int* cpre, TcCursor& c) {
  ++c.t;
  tc_settle(a, rpi, cpre, c);
}

__device__ __forceinline__ size_t tc_rec(const AttnArgs& a, int row, int head, int split) {
  return (((size_t)row * a.num_q_heads + head) * a.num_splits + split) * PREC;
}

// Empty records (m = -inf, l = 0) for the slots of an item: the combine kernel skips them.
__device__ __forceinline__ void tc_empty_record(const AttnArgs& a, const TcItem& it, int G, int tid) {
  if (tid < it.nr * G) {
    float* rec = a.partial + tc_rec(a, it.r0 + tid / G, it.kvh * G + tid % G, it.split);
    rec[D] = -INFINITY;
    rec[D + 1] = 0.f;
  }
}

template <int NS>
__global__ void __launch_bounds__(TC_THREADS, 1)
rows_partial_tc_kernel(const AttnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  using Smem = TcRowsSmem<NS>;
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.num_q_heads / a.num_kv_heads;
  const float qscale = a.sm_scale * 1.4426950408889634f;  // exp2 domain
  constexpr uint32_t tmem_cols = NS <= 16 ? 64 : 128;
  const int rpi = NS / G;
  const int* cpre = s.cpre;

  if (warp == 0) {
    tmem_alloc(&s.tmem_base, tmem_cols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.kfull, 1);
    mbar_init(&s.vfull[0], 1);
    mbar_init(&s.vfull[1], 1);
    mbar_init(&s.mma1, 1);
    mbar_init(&s.mma2, 1);
    fence_barrier_init();
  }
  {
    // Items before each sequence: thread t counts the row chunks of a contiguous block of
    // sequences, the block sums are scanned, and each thread writes its block's prefix.
    const int per = (a.num_seqs + TC_THREADS - 1) / TC_THREADS;
    const int s0 = min(a.num_seqs, tid * per), s1 = min(a.num_seqs, s0 + per);
    int sum = 0;
    for (int q = s0; q < s1; ++q) sum += (a.seq_start[q + 1] - a.seq_start[q] + rpi - 1) / rpi;
    s.tsum[tid] = sum;
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int i = 0; i < TC_THREADS; ++i) {
        const int v = s.tsum[i];
        s.tsum[i] = acc;
        acc += v;
      }
      s.tsum[TC_THREADS] = acc;
      s.cpre[a.num_seqs] = acc;
    }
    __syncthreads();
    int acc = s.tsum[tid];
    for (int q = s0; q < s1; ++q) {
      s.cpre[q] = acc;
      acc += (a.seq_start[q + 1] - a.seq_start[q] + rpi - 1) / rpi;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t t_s = tmem, t_o = tmem + NS;

  // Copy state (thread 0 only): cursors over the tile stream (K one tile ahead of the
  // consumer, V two) and the copies issued but not yet observed, per barrier.
  TcCursor kcur, vcur;
  int k_pend = 0, v_pend[2] = {0, 0};
  int k_uses = 0, v_uses[2] = {0, 0};
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(a.k_cache);
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(a.v_cache);
  auto issue = [&](const __nv_bfloat16* cache, uint8_t* dst, uint64_t* bar, const TcCursor& c) {
    const int pg0 = c.it.p0 + c.t * TC_PAGES;
    const int n = min(TC_PAGES, c.it.p1 - pg0);
    int page[TC_PAGES];
#pragma unroll
    for (int j = 0; j < TC_PAGES; ++j) page[j] = j < n ? __ldg(c.it.pt + pg0 + j) : 0;
    mbar_expect_tx(bar, n * BLOCK_BYTES);
#pragma unroll
    for (int j = 0; j < TC_PAGES; ++j)
      if (j < n) bulk_load(dst + j * BLOCK_BYTES, cache + kv_offset(a, page[j], c.it.kvh), BLOCK_BYTES, bar);
  };
  if (tid == 0) {
    tc_start(a, rpi, cpre, kcur);
    if (kcur.valid) {
      issue(kc, s.k, &s.kfull, kcur);
      k_pend = 1;
      tc_advance(a, rpi, cpre, kcur);
    }
    tc_start(a, rpi, cpre, vcur);
    for (int b = 0; b < 2 && vcur.valid; ++b) {
      issue(vc, s.v[b], &s.vfull[b], vcur);
      v_pend[b] = 1;
      tc_advance(a, rpi, cpre, vcur);
    }
  }

  bool ok = true;
  int f = 0;  // position in the tile stream: barrier phases and the V buffer
  int j = 0;
  TcItem it;
  for (; tc_item(a, blockIdx.x + j * gridDim.x, rpi, cpre, it); ++j) {
    // ---- item start: running max / sum, each slot's causal length and the Q slots
    // (slot = row * G + head; unused slots stay zero).  The previous item's products and
    // record reads are done.
    const int nslots = it.nr * G;
    if (tid < NS) {
      s.m[tid] = -INFINITY;
      s.l[tid] = 0.f;
      s.len[tid] = tid < nslots ? a.seq_lens[it.r0 + tid / G] : 0;
    }
    for (int i = tid; i < NS * 32; i += TC_THREADS) {
      const int h = i >> 5, pc = i & 31, c = pc >> 3, piece = pc & 7;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (h < nslots) {
        const __nv_bfloat16* qrow = static_cast<const __nv_bfloat16*>(a.q_out) +
                                    ((size_t)(it.r0 + h / G) * a.num_q_heads + it.kvh * G + h % G) * D;
        v = *reinterpret_cast<const uint4*>(qrow + pc * 8);
      }
      *reinterpret_cast<uint4*>(s.q[c] + h * 128 + ((piece ^ (h & 7)) << 4)) = v;
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    for (int t = 0; t < it.ntiles; ++t, ++f) {
      const int vb = f & 1;
      const int pg0 = it.p0 + t * TC_PAGES;
      const int n = min(TC_PAGES, it.p1 - pg0);
      if (n < TC_PAGES) {
        // Last, partial tile: zero the absent pages in both images (no copy targets them),
        // so the products see finite values there.
        for (int i = n * (BLOCK_BYTES / 16) + tid; i < TC_PAGES * (BLOCK_BYTES / 16); i += TC_THREADS) {
          reinterpret_cast<uint4*>(s.k)[i] = make_uint4(0, 0, 0, 0);
          reinterpret_cast<uint4*>(s.v[vb])[i] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_shared();
      }
      ok = mbar_wait(&s.kfull, (uint32_t)(k_uses & 1), a.err);
      if (!__syncthreads_and(ok)) break;
      if (tid == 0) {
        k_pend = 0;
        tc_fence_after();
        const uint32_t idesc = make_idesc_bf16(TC_KEYS, NS, 0, 0);
#pragma unroll
        for (int c = 0; c < TC_NCHUNK; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = make_smem_desc(smem_u32(s.k + c * 1024) + k * 32, 16, 4096, 2);
            const uint64_t bd = make_smem_desc(smem_u32(s.q[c]) + k * 32, 16, 1024, 2);
            mma_bf16(t_s, ad, bd, idesc, (c | k) ? 1u : 0u);
          }
        tc_commit(&s.mma1);
      }
      ++k_uses;
      ok = mbar_wait(&s.mma1, (uint32_t)(f & 1), a.err);
      if (!__syncthreads_and(ok)) break;
      tc_fence_after();
      // S is in TMEM: the K image is free, so the next tile's K copy (possibly the next
      // item's first) overlaps the rest of this tile.
      if (tid == 0 && kcur.valid) {
        issue(kc, s.k, &s.kfull, kcur);
        k_pend = 1;
        tc_advance(a, rpi, cpre, kcur);
      }
      // ---- online softmax: thread tid owns key tid of the tile
      uint32_t sr[NS];
#pragma unroll
      for (int c0 = 0; c0 < NS; c0 += 16) {
        uint32_t part[16];
        tmem_ld_32x32b_x16(t_s + c0 + lane_off, part);
#pragma unroll
        for (int h = 0; h < 16; ++h) sr[c0 + h] = part[h];
      }
      tmem_ld_wait();
      // Key tok counts for slot h when it lies in this split's pages (tok_end) and inside
      // the slot's causal length.
      const int tok = pg0 * PAGE + tid;
      const bool in_split = tok < it.tok_end;
      float sv[NS];
#pragma unroll
      for (int h = 0; h < NS; ++h)
        sv[h] = (in_split && tok < s.len[h]) ? __uint_as_float(sr[h]) * qscale : -INFINITY;
#pragma unroll
      for (int h = 0; h < NS; ++h) {
        const float v = warp_max(sv[h]);
        if (lane == 0) s.red_max[warp][h] = v;
      }
      __syncthreads();
      float mnew[NS];
#pragma unroll
      for (int h = 0; h < NS; ++h)
        mnew[h] = fmaxf(fmaxf(s.m[h], fmaxf(s.red_max[0][h], s.red_max[1][h])), fmaxf(s.red_max[2][h], s.red_max[3][h]));
      {
        const int chunk = tid >> 6, within = tid & 63, piece = within >> 3, sub = (within & 7) * 2;
#pragma unroll
        for (int h = 0; h < NS; ++h) {
          const float pv = sv[h] == -INFINITY ? 0.f : exp2f(sv[h] - mnew[h]);
          const __nv_bfloat16 pb = __float2bfloat16_rn(pv);
          *reinterpret_cast<__nv_bfloat16*>(s.p[chunk] + h * 128 + ((piece ^ (h & 7)) << 4) + sub) = pb;
          const float sum = warp_sum(__bfloat162float(pb));
          if (lane == 0) s.red_sum[warp][h] = sum;
        }
      }
      fence_proxy_async_shared();
      __syncthreads();
      if (tid < NS) {
        const int h = tid;
        const float mo = s.m[h];
        const float rr = mo == -INFINITY ? 0.f : exp2f(mo - mnew[h]);
        s.l[h] = s.l[h] * rr + (s.red_sum[0][h] + s.red_sum[1][h] + s.red_sum[2][h] + s.red_sum[3][h]);
        s.m[h] = mnew[h];
        s.r[h] = rr;
      }
      __syncthreads();
      if (t > 0) {  // rescale the running O^T (TMEM lane = head dim, column = query slot)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int c0 = 0; c0 < NS; c0 += 16) {
            uint32_t o[16];
            tmem_ld_32x32b_x16(t_o + mt * NS + c0 + lane_off, o);
            tmem_ld_wait();
#pragma unroll
            for (int h = 0; h < 16; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * s.r[c0 + h]);
            tmem_st_32x32b_x16(t_o + mt * NS + c0 + lane_off, o);
          }
        tmem_st_wait();
      }
      ok = mbar_wait(&s.vfull[vb], (uint32_t)(v_uses[vb] & 1), a.err);
      if (ok && !in_split && tok < (pg0 + n) * PAGE) {
        // Cache rows past the context inside a loaded page: zero them (P is 0 there).
        const int r = tid & 15;
        uint8_t* blk = s.v[vb] + (tid >> 4) * BLOCK_BYTES + (r >> 3) * 4096 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < TC_NCHUNK; ++c) {
          uint4* rowp = reinterpret_cast<uint4*>(blk + c * 1024);
#pragma unroll
          for (int q = 0; q < 8; ++q) rowp[q] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_shared();
      }
      tc_fence_before();
      if (!__syncthreads_and(ok)) break;
      if (tid == 0) {
        v_pend[vb] = 0;
        tc_fence_after();
        const uint32_t idesc2 = make_idesc_bf16(128, NS, 1, 0);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t ad = make_smem_desc(smem_u32(s.v[vb] + 2 * mt * 1024) + ks * BLOCK_BYTES, 1024, 4096, 2);
            const uint64_t bd = make_smem_desc(smem_u32(s.p[ks >> 2]) + (ks & 3) * 32, 16, 1024, 2);
            mma_bf16(t_o + mt * NS, ad, bd, idesc2, (t > 0 || ks > 0) ? 1u : 0u);
          }
        tc_commit(&s.mma2);
      }
      ++v_uses[vb];
      ok = mbar_wait(&s.mma2, (uint32_t)(f & 1), a.err);
      if (!__syncthreads_and(ok)) break;
      tc_fence_after();
      if (tid == 0 && vcur.valid) {  // this V image is free: the tile two ahead in the stream
        issue(vc, s.v[vb], &s.vfull[vb], vcur);
        v_pend[vb] = 1;
        tc_advance(a, rpi, cpre, vcur);
      }
    }
    if (!ok) break;
    // ---- item end: the record (o, m, l) of every used slot
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int c0 = 0; c0 < NS; c0 += 16) {
        if (c0 >= nslots) break;
        uint32_t o[16];
        if (it.ntiles > 0) {
          tmem_ld_32x32b_x16(t_o + mt * NS + c0 + lane_off, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int h = 0; h < 16; ++h) o[h] = 0u;
        }
        const int dim = mt * 128 + tid;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const int sl = c0 + h;
          if (sl >= nslots) break;
          a.partial[tc_rec(a, it.r0 + sl / G, it.kvh * G + sl % G, it.split) + dim] = __uint_as_float(o[h]);
        }
      }
    if (tid < nslots) {
      float* rec = a.partial + tc_rec(a, it.r0 + tid / G, it.kvh * G + tid % G, it.split);
      rec[D] = s.m[tid];
      rec[D + 1] = s.l[tid];
    }
    // The next item's products overwrite S and O, and its set-up rewrites m / l / len.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (!ok) {
    // Abort (the error word is set): still write empty records (m = -inf, l = 0) for this
    // item and every later one of this CTA, so the combine kernel skips them instead of
    // reading whatever an earlier call left in the scratch buffer.
    for (; tc_item(a, blockIdx.x + j * gridDim.x, rpi, cpre, it); ++j) tc_empty_record(a, it, G, tid);
    // Let every copy still in flight land before the CTA releases shared memory.
    if (tid == 0) {
      if (k_pend) mbar_wait(&s.kfull, (uint32_t)(k_uses & 1), nullptr);
      for (int b = 0; b < 2; ++b)
        if (v_pend[b]) mbar_wait(&s.vfull[b], (uint32_t)(v_uses[b] & 1), nullptr);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, tmem_cols);
}

// One CTA (256 threads, thread = dim) per (row, q head): merge splits, normalise,
// apply sigmoid(gate), write bf16 and/or MXFP8.
__global__ void decode_combine_kernel(const AttnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int row = blockIdx.x, qh = blockIdx.y, d = threadIdx.x;
  const float* rec = a.partial + ((size_t)row * a.num_q_heads + qh) * a.num_splits * PREC;
  float m = -INFINITY;
  for (int s = 0; s < a.num_splits; ++s) m = fmaxf(m, rec[s * PREC + D]);
  float l = 0.f, o = 0.f;
  for (int s = 0; s < a.num_splits; ++s) {
    const float ms = rec[s * PREC + D];
    if (ms == -INFINITY) continue;
    const float sc = exp2f(ms - m);
    l += rec[s * PREC + D + 1] * sc;
    o += rec[s * PREC + d] * sc;
  }
  const float attn = l > 0.f ? o / l : 0.f;
  const float g = __bfloat162float(static_cast<const __nv_bfloat16*>(a.gate_out)[((size_t)row * a.num_q_heads + qh) * D + d]);
  const float y = bfr(bfr(attn) * sigmoidf_(g));
  const int width = a.num_q_heads * D;
  const int col = qh * D + d;
  if (a.out_bf16 != nullptr) static_cast<__nv_bfloat16*>(a.out_bf16)[(size_t)row * width + col] = __float2bfloat16_rn(y);
  if (a.out_q != nullptr) {
    const float amax = warp_max(fabsf(y));
    const uint8_t code = mx_scale_e8m0(amax);
    a.out_q[(size_t)row * width + col] = f32_to_e4m3(y * mx_inv_scale(code));
    if ((d & 31) == 0) {
      const int kb = col >> 5;
      a.out_sf[((size_t)(row >> 7) * (width >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] = code;
    }
  }
}

}  // namespace attn
}  // namespace zs

extern "C" int zs_attn_prologue(const AttnArgs* args, cudaStream_t stream) {
  const AttnArgs& a = *args;
  if (a.head_dim != zs::attn::D || a.rotary_dim % 16 != 0 || a.rotary_dim > a.head_dim) return -1;
  if (a.rows == 0) return 0;
  zs_launch(zs::attn::prologue_kernel, a.rows, 256, 0, stream, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int zs_attn_decode(const AttnArgs* args, cudaStream_t stream) {
  const AttnArgs& a = *args;
  if (a.head_dim != zs::attn::D || a.num_kv_heads <= 0 || a.num_q_heads % a.num_kv_heads != 0) return -1;
  const int group = a.num_q_heads / a.num_kv_heads;
  if (a.num_splits < 1 || a.partial == nullptr || a.page_size != zs::attn::PAGE) return -1;
  if (a.rows == 0) return 0;
  dim3 g1(a.rows, a.num_kv_heads, a.num_splits);
  // impl 0 picks: tensor cores from 4 query heads per kv head; smaller groups (a GQA group
  // split over many ranks) stay on the SIMT kernel, which runs one warp per head.  impl 1
  // forces the SIMT kernel, impl 2 the tensor-core kernels for any group up to 16.
  const bool tc = (a.impl == 0 && group >= 4 && group <= zs::attn::TC_N) || (a.impl == 2 && group <= zs::attn::TC_N);
  if (tc) {
    if (a.seq_start != nullptr && a.num_seqs > 0 && a.num_seqs <= zs::attn::TC_MAX_SEQS) {
      // Rows grouped by sequence: multi-row items of 32 query slots, one CTA per item
      // (the item count is bounded above: every sequence adds at most one partial chunk).
      const int rpi = zs::attn::TC_NMR / group;
      const long long items = ((long long)a.rows / rpi + a.num_seqs) * a.num_kv_heads * a.num_splits;
      const size_t smem = sizeof(zs::attn::TcRowsSmem<zs::attn::TC_NMR>) + 1024;
      auto kern = zs::attn::rows_partial_tc_kernel<zs::attn::TC_NMR>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      zs_launch(kern, (int)items, zs::attn::TC_THREADS, smem, stream, a);
    } else {
      const size_t smem = sizeof(zs::attn::TcSmem) + 1024;
      cudaFuncSetAttribute(zs::attn::decode_partial_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      zs_launch(zs::attn::decode_partial_tc_kernel, g1, zs::attn::TC_THREADS, smem, stream, a);
    }
    dim3 g2(a.rows, a.num_q_heads);
    zs_launch(zs::attn::decode_combine_kernel, g2, zs::attn::D, 0, stream, a);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
  if (group > 8) return -1;
  const size_t smem = sizeof(zs::attn::DecSmem) + 128;
  cudaFuncSetAttribute(zs::attn::decode_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  zs_launch(zs::attn::decode_partial_kernel, g1, group * 32, smem, stream, a);
  dim3 g2(a.rows, a.num_q_heads);
  zs_launch(zs::attn::decode_combine_kernel, g2, zs::attn::D, 0, stream, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Varlen prefill: identical math with per-row causal context lengths (seq_lens must
// hold position + 1 for every row); the caller runs the prologue for all rows first.
extern "C" int zs_attn_prefill(const AttnArgs* args, cudaStream_t stream) {
  return zs_attn_decode(args, stream);
}

// ---------------------------------------------------------------------------------------
// Allocation-free decode entry point (no counterpart in the reference).
//
// zs_attn_decode_noalloc computes the same gated paged attention as zs_attn_decode, but the
// caller passes no split-KV scratch buffer: the per-split partial records live in one fixed
// device array that is part of this library's image.  It serves callers that cannot allocate
// device memory at the point of the call: a host runtime whose device allocator belongs to
// another framework (so a private cudaMalloc would fragment or exceed its budget), a plugin
// that must not change the process's memory footprint after start-up, or plain C code that
// holds only raw device pointers and no allocator at all.
//
// Limit: the array holds ZS_ATTN_NOALLOC_SCRATCH_FLOATS floats (8 MiB).  A call needs
// rows * num_q_heads * num_splits * 260 floats; above that it returns -3 and launches nothing.
// Sharing: every call on a device uses the same array, so calls that overlap in time (two
// streams, or two host threads without ordering between their streams) race on it; issue
// them on one stream.  Nothing in the array has to start at zero: every split record the
// combine step reads is written earlier in the same call (an aborted split writes an empty
// record), so contents left by a previous call are never mixed in.
// Set-up: the first call on each device looks up the array's address with that device
// current and caches it; make the first call on a device before any stream capture.
static __device__ __align__(256) float g_attn_noalloc_scratch[ZS_ATTN_NOALLOC_SCRATCH_FLOATS];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {};
}  // namespace

extern "C" int zs_attn_decode_noalloc(const AttnArgs* args, cudaStream_t stream) {
  const AttnArgs& in = *args;
  // Size check without overflow: divide the limit by each factor in turn instead of
  // multiplying the caller's ints together.
  const size_t limit = (size_t)ZS_ATTN_NOALLOC_SCRATCH_FLOATS;
  bool fits = in.rows >= 0 && in.num_q_heads >= 0 && in.num_splits >= 0;
  if (fits && in.rows > 0 && in.num_q_heads > 0 && in.num_splits > 0) {
    size_t room = limit / zs::attn::PREC;
    room /= (size_t)in.rows;
    room /= (size_t)in.num_q_heads;
    fits = (size_t)in.num_splits <= room;
  }
  if (!fits) {
    fprintf(stderr, "zs_attn_decode_noalloc: rows %d x q heads %d x splits %d x %d floats exceed the fixed "
            "scratch of %zu floats\n", in.rows, in.num_q_heads, in.num_splits, zs::attn::PREC, limit);
    return -3;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -4;
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_attn_noalloc_scratch) != cudaSuccess || p == nullptr) return -4;
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_noalloc_ptr[dev];
  }
  AttnArgs a = in;
  a.partial = scratch;
  return zs_attn_decode(&a, stream);
}

// Block-scaled MXFP8 GEMM for sm_100a: tcgen05.mma.kind::mxf8f6f4.block_scale with
// TMA-fed shared-memory operands and TMEM accumulators.
//
// Orientation ("swap-AB"): the weight matrix is the MMA's M side (128 output features
// per tile) and the tokens are the N side (16..BN per pass), so decode batches of a
// handful of tokens per expert still issue full-height MMAs and the kernel streams the
// weights at HBM rate.  One persistent CTA per SM walks a static list of work items
// (group, 128-feature tile, BN-token chunk, K split).  Roles inside a CTA:
//   warps 0-3 : epilogue (TMEM -> registers -> fused op -> global)
//   warp 4    : TMA / bulk-copy producer
//   warp 5    : MMA issuer (one thread) + scale-factor TMEM staging (tcgen05.cp)
// Accumulators are double-buffered in TMEM so the epilogue of tile i overlaps the
// main loop of tile i+1.  Each pipeline stage holds two K tiles (KT = 2).  Instantiations:
// BN=128 with 3 stages for prefill-sized token counts, BN=32 with 4 stages for decode,
// where each expert sees a few tokens and the kernel is a weight stream that wants as many
// bytes in flight as shared memory allows; the MXFP4 variants use 2 and 3 stages (their
// packed staging buffers take the rest).
//
// Operand formats (all produced by this library's quantizers):
//   A  weights      e4m3 [G * Npad, K], K contiguous; Npad % 128 == 0, K % 128 == 0
//   SFA weight sf   e8m0 [G, Npad/128, K/128, 512]   (128-row x 4-block atoms)
//   B  activations  e4m3 [rows, K] in per-group segments starting at multiples of 128
//   SFB act sf      e8m0 [rows/128, K/128, 512]
// Atom byte layout: row r = r0 + 32*r1 (r0 < 32) and 32-wide K block j (j < 4) live
// at byte r0*16 + r1*4 + j, which is what tcgen05.cp.32x128b.warpx4 expects: TMEM
// column r1 holds rows 32*r1..32*r1+31, so a 32-token chunk that starts 32*j rows
// into an atom points the MMA's B-scale address at column j of the staged atom.
//
// Split-K, two forms.  (1) k_splits (dense, fp32 output): item (m, chunk, ks) covers K
// tiles [ks*kps, (ks+1)*kps) and stores its partial at out + ks*split_stride; the
// consumer sums the splits in a fixed order.  (2) fix_splits (any mode): the splits of
// one output tile run on different CTAs, publish fp32 partials to a workspace and bump
// a per-tile counter; the CTA that completes the tile sums the partials in split order
// (deterministic) and runs the epilogue.  A single CTA streams only ~90 GB/s from HBM,
// so small GEMMs need the extra CTAs to reach full bandwidth.
//
// Reference parity: replaces the reference's Triton grouped MoE GEMMs and skinny
// linears (worker/zstep_worker/kernels_sm120/qwen35_ops.py:1226-1438) and the
// b12x MXFP8 linears (kernels_sm120/b12x_dsv41.py:370) with one tcgen05 kernel.
#include "peer.cuh"
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace gemm {

constexpr int BM = 128;   // weight rows per tile (MMA M)
constexpr int BK = 128;   // K elements (bytes) per stage = one 128B swizzle span
constexpr int A_BYTES = BM * BK;
constexpr int SF_BYTES = 512;
constexpr int kMaxGroups = 520;  // grouped mode: per-group tables are staged in smem
constexpr int kMaxFixSplits = 8; // in-kernel split-K factor limit

template <int BN, int STAGES, bool FP4 = false>
struct Cfg {
  // Each pipeline stage holds KT consecutive K tiles, so one bulk copy moves 32 KiB of
  // weights and one 3-D TMA box both tiles of activations: the producer issues half as
  // many copy instructions (each costs ~50-90 ns of issue time on one SM).
  static constexpr int KT = 2;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int ACC_COLS = BN;              // fp32 accumulator columns per buffer
  // Scale factors are double-buffered by K-tile parity (8 columns per buffer: SFA 4 +
  // SFB 4) so staging the next tile's scales does not wait for this tile's MMAs.
  static constexpr int SFA_COL = 2 * BN;           // + 8 * (kt & 1), 4 columns
  static constexpr int SFB_COL = 2 * BN + 4;       // + 8 * (kt & 1), 4 columns
  static constexpr int TMEM_COLS = (2 * BN + 16) <= 128 ? 128 : ((2 * BN + 16) <= 256 ? 256 : 512);
  static constexpr int A4_BYTES = FP4 ? A_BYTES / 2 : 16;  // packed e2m1 staging per tile
  static constexpr int THREADS = FP4 ? 320 : 192;          // + 4 converter warps for FP4
  struct Smem {
    uint8_t a[STAGES][KT][A_BYTES];
    uint8_t b[STAGES][KT][B_BYTES];
    uint8_t sfa[STAGES][KT][SF_BYTES];
    uint8_t sfb[STAGES][KT][SF_BYTES];
    float xch[32][65];              // epilogue exchange (gate/up pairing, then the transpose)
    unsigned long long red[4][32];  // epilogue exchange (argmax)
    int g_prefix[kMaxGroups + 1];   // grouped mode: chunk prefix, offsets, counts
    int g_offset[kMaxGroups];
    int g_count[kMaxGroups];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t conv[STAGES];          // FP4: the converter warps widened stage's weights
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    int fix_last;                   // split-K: this CTA completed the current tile
    // FP4 staging last, so the swizzled operand buffers above keep their 1024-byte
    // alignment in every instantiation.
    alignas(1024) uint8_t a4[FP4 ? STAGES : 1][KT][A4_BYTES];
  };
};

struct Item {
  int g, m, c, count, seg_off, kt0, kt1, ks;
  int tile;  // output tile id (split-K bookkeeping)
};

// Work item `idx`.  Grouped mode reads the per-group tables staged in shared memory
// (pre/off/cnt), so the per-item lookup is a short binary search without global loads.
template <int BN>
__device__ __forceinline__ bool get_item(const GemmMxf8Args& p, int idx, Item& it, const int* pre,
                                         const int* off, const int* cnt) {
  const int m_tiles = p.n_pad / BM;
  const int k_tiles = p.k / BK;
  if (p.chunk_prefix == nullptr) {
    const int chunks = (p.m_rows + BN - 1) / BN;
    const int splits = p.k_splits > 1 ? p.k_splits : (p.fix_splits > 1 ? p.fix_splits : 1);
    if (idx >= chunks * m_tiles * splits) return false;
    it.ks = idx % splits;
    const int rest = idx / splits;
    it.tile = rest;
    it.g = 0;
    it.m = rest % m_tiles;
    it.c = rest / m_tiles;
    it.seg_off = 0;
    it.count = min(BN, p.m_rows - it.c * BN);
    const int kps = (k_tiles + splits - 1) / splits;
    it.kt0 = it.ks * kps;
    it.kt1 = min(k_tiles, it.kt0 + kps);
    return true;
  }
  const int S = p.fix_splits > 1 ? p.fix_splits : 1;
  const int total_chunks = pre[p.groups];
  // With last_mt > 0 the last group's chunks cover only tiles [last_m0, last_m0 + last_mt).
  const int pre_last = p.last_mt > 0 ? pre[p.groups - 1] : total_chunks;
  const int full_tiles = pre_last * m_tiles;
  const int total_tiles = full_tiles + (total_chunks - pre_last) * (p.last_mt > 0 ? p.last_mt : 0);
  if (idx >= total_tiles * S) return false;
  const int t = idx / S;
  if (S > 1 && t >= p.max_tiles) return false;  // workspace too small: the producer reports it
  it.ks = idx % S;
  it.tile = t;
  int chunk;
  if (t < full_tiles) {
    chunk = t / m_tiles;
    it.m = t % m_tiles;
  } else {
    chunk = pre_last + (t - full_tiles) / p.last_mt;
    it.m = p.last_m0 + (t - full_tiles) % p.last_mt;
  }
  int lo = 0, hi = p.groups;  // largest g with prefix[g] <= chunk
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pre[mid] <= chunk) lo = mid; else hi = mid;
  }
  it.g = lo;
  it.c = chunk - pre[lo];
  it.seg_off = off[lo];
  it.count = min(BN, cnt[lo] - it.c * BN);
  const int kps = k_tiles / S;
  it.kt0 = it.ks * kps;
  it.kt1 = it.kt0 + kps;
  return true;
}

// Accumulator columns [col0, col0 + ncols) (ncols <= 32) of this thread's row.  Without
// split-K they come straight from TMEM (col0 is a multiple of 32 then); with split-K they
// are the sum of every split's fp32 partial, in split order, from the workspace.
template <int BN>
__device__ __forceinline__ void load_cols(uint32_t t_base, const GemmMxf8Args& p, const Item& it, int S, int col0,
                                          int ncols, int row_in_tile, float (&v)[32]) {
  if (S == 1) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_base + col0, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = 0.f;
  const float* base = p.ws + (size_t)it.tile * S * (BN * BM) + (size_t)col0 * BM + row_in_tile;
  for (int q = 0; q < S; ++q) {
    const float* w = base + (size_t)q * (BN * BM);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncols) v[j] += __ldcg(w + j * BM);
  }
}

__device__ __forceinline__ int sem_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t phase, int* err,
                                              volatile int* abort_flag) {
  for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
    if (*abort_flag) return false;
    if (i > 64) __nanosleep(64);
  }
  report_error(err, kErrMbarTimeout);
  *abort_flag = 1;
  return false;
}

// Widen 8 packed e2m1 values (one 32-bit word, element i in nibble i) to 8 e4m3 bytes:
// a byte permute picks each magnitude from an 8-entry table of the e4m3 images of
// 0, 0.5, 1, 1.5, 2, 3, 4, 6; a second permute turns each sign bit into 0x00 / 0x80.
__device__ __forceinline__ uint2 widen_e2m1x8(uint32_t w) {
  const uint32_t lo = 0x3C383000u, hi = 0x4C484440u;
  const uint32_t m0 = __byte_perm(lo, hi, w & 0x7777u);
  const uint32_t s0 = __byte_perm(0x00008000u, 0u, (w >> 3) & 0x1111u);
  const uint32_t m1 = __byte_perm(lo, hi, (w >> 16) & 0x7777u);
  const uint32_t s1 = __byte_perm(0x00008000u, 0u, (w >> 19) & 0x1111u);
  return make_uint2(m0 | s0, m1 | s1);
}

template <int BN, int STAGES, bool FP4>
__global__ void __launch_bounds__(Cfg<BN, STAGES, FP4>::THREADS, 1)
gemm_mxf8_kernel(const __grid_constant__ CUtensorMap tmap_a,
                 const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_b_full,
                 const GemmMxf8Args p) {
  using C = Cfg<BN, STAGES, FP4>;
  using Smem = typename C::Smem;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = warp_id();
  const int lane = lane_id();
  volatile int* abort_flag = &s.abort_flag;
  const int k_tiles = p.k / BK;

  // Set-up that reads nothing a predecessor kernel writes runs before the dependency wait,
  // so under programmatic dependent launch it overlaps the previous kernel's tail.
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
      mbar_init(&s.conv[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 4);
    }
    mbar_init(&s.drain, 1);
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_b_full);
  }
  __syncthreads();  // barriers initialised before the producer arms them
  // Weights never change during a step, so in dense mode the producer starts streaming
  // the first item's weight stages (and their scales) before the dependency wait; the
  // activation half of those stages is issued after it.  `pre` stages are armed here.
  int pre = 0;
  auto stage_bytes = [&](const Item& it, int n_sub) -> uint32_t {
    const int n16 = (it.count + 15) >> 4;
    const bool full_b = n16 * 16 == BN;
    const int a_bytes = FP4 ? C::A4_BYTES : A_BYTES;
    return n_sub * (a_bytes + 2 * SF_BYTES) + (full_b ? C::KT : n_sub) * n16 * 16 * BK;
  };
  auto issue_a = [&](const Item& it, int st, int kt, int n_sub) {
    const int a_row = it.g * p.n_pad + it.m * BM;
    if (FP4) {  // packed e2m1 tiles into the staging buffer; the converter warps widen them
      bulk_load(s.a4[st][0], p.a + ((size_t)(a_row / BM) * k_tiles + kt) * C::A4_BYTES, n_sub * C::A4_BYTES,
                &s.full[st]);
    } else if (p.a_tiled) {  // pre-swizzled contiguous tiles: one plain bulk copy
      bulk_load(s.a[st][0], p.a + ((size_t)(a_row / BM) * k_tiles + kt) * A_BYTES, n_sub * A_BYTES, &s.full[st]);
    } else {
      for (int j = 0; j < n_sub; ++j) tma_load_2d(s.a[st][j], &tmap_a, &s.full[st], (kt + j) * BK, a_row);
    }
    const uint8_t* sfa_src = p.sfa + ((size_t)(it.g * (p.n_pad / BM) + it.m) * k_tiles) * SF_BYTES;
    bulk_load(s.sfa[st][0], sfa_src + (size_t)kt * SF_BYTES, n_sub * SF_BYTES, &s.full[st]);
  };
  // Activation half of a stage (after the dependency wait).
  auto issue_b = [&](const Item& it, int st, int kt, int n_sub, int n16, int b_row, const uint8_t* sfb_src) {
    if (n16 * 16 == BN) {
      tma_load_3d(s.b[st][0], &tmap_b_full, &s.full[st], 0, b_row, kt);  // one BN-row x KT box
    } else {
      for (int t = 0; t < n_sub; ++t)
        for (int j = 0; j < n16; ++j)
          tma_load_2d(s.b[st][t] + j * 16 * BK, &tmap_b, &s.full[st], (kt + t) * BK, b_row + j * 16);
    }
    bulk_load(s.sfb[st][0], sfb_src + (size_t)kt * SF_BYTES, n_sub * SF_BYTES, &s.full[st]);
  };
  if (warp == 4 && lane == 0 && p.chunk_prefix == nullptr) {
    Item it0;
    if (get_item<BN>(p, blockIdx.x, it0, nullptr, nullptr, nullptr)) {
      for (int kt = it0.kt0; kt < it0.kt1 && pre < STAGES; kt += C::KT, ++pre) {
        const int n_sub = min(C::KT, it0.kt1 - kt);
        mbar_expect_tx(&s.full[pre], stage_bytes(it0, n_sub));
        issue_a(it0, pre, kt, n_sub);
      }
    }
  }
  pdl_wait();  // predecessor kernel done: its outputs (activations, group tables) are visible
  pdl_trigger();
  if (p.chunk_prefix != nullptr) {
    for (int g = threadIdx.x; g <= p.groups; g += C::THREADS) s.g_prefix[g] = __ldg(p.chunk_prefix + g);
    for (int g = threadIdx.x; g < p.groups; g += C::THREADS) {
      s.g_offset[g] = __ldg(p.group_offset + g);
      s.g_count[g] = __ldg(p.group_count + g);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t issued = 0;
      Item it;
      for (int idx = blockIdx.x; get_item<BN>(p, idx, it, s.g_prefix, s.g_offset, s.g_count) && !*abort_flag; idx += gridDim.x) {
        const int n16 = (it.count + 15) >> 4;
        const int b_row = it.seg_off + it.c * BN;
        const uint8_t* sfb_src = p.sfb + ((size_t)(b_row / BM) * k_tiles) * SF_BYTES;
        for (int kt = it.kt0; kt < it.kt1; kt += C::KT) {
          const int n_sub = min(C::KT, it.kt1 - kt);
          const int st = issued % STAGES;
          const uint32_t ph = ((issued / STAGES) & 1) ^ 1;
          if (issued >= STAGES && !wait_or_abort(&s.empty[st], ph, p.err, abort_flag)) break;
          // A full-height B box spans KT tiles (a tile past the end of K is zero-filled);
          // short chunks load n16 16-row boxes per tile.
          if ((int)issued >= pre) {  // else: armed, weights requested before the dependency wait
            mbar_expect_tx(&s.full[st], stage_bytes(it, n_sub));
            issue_a(it, st, kt, n_sub);
          }
          issue_b(it, st, kt, n_sub, n16, b_row, sfb_src);
          ++issued;
        }
      }
      if ((int)issued < pre) {
        // Aborted before reaching every armed stage: complete their activation halves too,
        // so each copy in flight finishes its barrier and the drain below can see it land.
        Item it0;
        get_item<BN>(p, blockIdx.x, it0, nullptr, nullptr, nullptr);
        for (; (int)issued < pre; ++issued) {
          const int kt = it0.kt0 + (int)issued * C::KT;
          const int b_row = it0.seg_off + it0.c * BN;
          issue_b(it0, issued, kt, min(C::KT, it0.kt1 - kt), (it0.count + 15) >> 4, b_row,
                  p.sfb + ((size_t)(b_row / BM) * k_tiles) * SF_BYTES);
        }
      }
      if (blockIdx.x == 0 && p.fix_splits > 1 && p.chunk_prefix != nullptr &&
          s.g_prefix[p.groups] * (p.n_pad / BM) > p.max_tiles)
        report_error(p.err, kErrBadShape);  // split-K workspace smaller than the tile count
      // Drain: wait (bounded) until every fill this thread issued has landed, so no
      // copy is still writing shared memory when the CTA exits.
      const uint32_t first = issued > STAGES ? issued - STAGES : 0;
      for (uint32_t q = first; q < issued; ++q) {
        if (!mbar_wait(&s.full[q % STAGES], (q / STAGES) & 1, nullptr)) {
          report_error(p.err, kErrDrainTimeout);
          break;
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the loop (lane 0 issues the tcgen05 ops); for 32-token
    // chunks that start 32*j0 rows into a scale atom, the warp first moves each
    // line's 4 scale bytes of rows 32*j0.. to the line's first word, so the staged
    // scales always start at an aligned TMEM column.
    uint32_t consumed = 0, sub_count = 0;
    uint32_t acc_uses[2] = {0, 0};
    int local = 0;
    Item it;
    for (int idx = blockIdx.x; get_item<BN>(p, idx, it, s.g_prefix, s.g_offset, s.g_count) && !*abort_flag; idx += gridDim.x, ++local) {
      const int buf = local & 1;
      // Every lane waits itself, so each observes the barrier (acquire) before touching
      // the staged data.
      bool ok = wait_or_abort(&s.acc_empty[buf], (acc_uses[buf] & 1) ^ 1, p.err, abort_flag);
      if (!__all_sync(0xffffffff, ok)) break;
      ++acc_uses[buf];
      tc_fence_after();
      const uint32_t n_mma = ((it.count + 15) >> 4) << 4;
      const uint32_t d_tmem = tmem + buf * C::ACC_COLS;
      const int j0 = ((it.seg_off + it.c * BN) & 127) >> 5;  // nonzero only when BN < 128
      for (int kt = it.kt0; kt < it.kt1; kt += C::KT) {
        const int n_sub = min(C::KT, it.kt1 - kt);
        const int st = consumed % STAGES;
        ok = wait_or_abort(&s.full[st], (consumed / STAGES) & 1, p.err, abort_flag);
        if (FP4 && ok) ok = wait_or_abort(&s.conv[st], (consumed / STAGES) & 1, p.err, abort_flag);
        if (!__all_sync(0xffffffff, ok)) {
          ok = false;
          break;
        }
        for (int j = 0; j < n_sub; ++j) {
          if (BN < 128 && j0 != 0) {
            uint32_t* line = reinterpret_cast<uint32_t*>(s.sfb[st][j] + lane * 16);
            line[0] = line[j0];
            fence_proxy_async_shared();
            __syncwarp();
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t sf_off = (sub_count & 1) * 8;
            tmem_cp_32x128b_warpx4(tmem + C::SFA_COL + sf_off, make_smem_desc(smem_u32(s.sfa[st][j]), 0, 128, 0));
            tmem_cp_32x128b_warpx4(tmem + C::SFB_COL + sf_off, make_smem_desc(smem_u32(s.sfb[st][j]), 0, 128, 0));
            const uint32_t a_base = smem_u32(s.a[st][j]);
            const uint32_t b_base = smem_u32(s.b[st][j]);
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
              const uint64_t adesc = make_smem_desc(a_base + kb * 32, 16, 1024, 2);
              const uint64_t bdesc = make_smem_desc(b_base + kb * 32, 16, 1024, 2);
              const uint32_t idesc = make_idesc_mxf8(BM, n_mma, kb, kb);
              mma_mxf8(d_tmem, adesc, bdesc, idesc, (tmem + C::SFA_COL + sf_off) | (uint32_t(kb) << 30),
                       (tmem + C::SFB_COL + sf_off) | (uint32_t(kb) << 30), (kt + j > it.kt0 || kb > 0) ? 1u : 0u);
            }
          }
          __syncwarp();
          ++sub_count;
        }
        if (lane == 0) tc_commit(&s.empty[st]);
        __syncwarp();
        ++consumed;
      }
      if (!ok) break;
      if (lane == 0) tc_commit(&s.acc_full[buf]);
      __syncwarp();
    }
    // Make sure no MMA is still running before TMEM is released.
    if (lane == 0) {
      tc_commit(&s.drain);
      if (!mbar_wait(&s.drain, 0, nullptr)) report_error(p.err, kErrDrainTimeout);
    }
    __syncwarp();
  } else if (FP4 && warp >= 6) {
    // ------------------------------------------------------------------ FP4 converters
    // Walk the same stage sequence as the MMA warp: once a stage's copies landed, widen
    // its packed weight tiles into the swizzled e4m3 image the MMA reads (piece c of row
    // r at piece c ^ (r % 8)), make the writes visible to the tensor core, and arrive.
    const int ct = threadIdx.x - 192;
    uint32_t consumed = 0;
    bool ok = true;
    Item it;
    for (int idx = blockIdx.x; ok && get_item<BN>(p, idx, it, s.g_prefix, s.g_offset, s.g_count) && !*abort_flag;
         idx += gridDim.x) {
      for (int kt = it.kt0; kt < it.kt1; kt += C::KT) {
        const int n_sub = min(C::KT, it.kt1 - kt);
        const int st = consumed % STAGES;
        ok = wait_or_abort(&s.full[st], (consumed / STAGES) & 1, p.err, abort_flag);
        if (!__all_sync(0xffffffff, ok)) {
          ok = false;
          break;
        }
        for (int j = 0; j < n_sub; ++j) {
          const uint8_t* src = s.a4[st][j];
          uint8_t* dst = s.a[st][j];
#pragma unroll 4
          for (int task = ct; task < BM * 8; task += 128) {
            const int r = task >> 3, c = task & 7;
            const uint2 v = *reinterpret_cast<const uint2*>(src + r * 64 + c * 8);
            const uint2 w0 = widen_e2m1x8(v.x), w1 = widen_e2m1x8(v.y);
            *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(w0.x, w0.y, w1.x, w1.y);
          }
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.conv[st]);
        ++consumed;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    // Each thread owns one accumulator row (a weight feature) and walks the token
    // columns 32 at a time.  With in-kernel split-K the CTA first publishes its fp32
    // partial; only the CTA that completes the tile sums all partials (fixed split
    // order, so the result does not depend on arrival order) and runs the epilogue.
    const int q = warp;  // TMEM subpartition (lanes 32q .. 32q+31)
    const int row_in_tile = q * 32 + lane;
    const int S = p.fix_splits > 1 ? p.fix_splits : 1;
    const long long split_off = p.k_splits > 1 ? 1 : 0;
    uint32_t acc_uses[2] = {0, 0};
    int local = 0;
    Item it;
    for (int idx = blockIdx.x; get_item<BN>(p, idx, it, s.g_prefix, s.g_offset, s.g_count); idx += gridDim.x, ++local) {
      const int buf = local & 1;
      if (!wait_or_abort(&s.acc_full[buf], acc_uses[buf] & 1, p.err, abort_flag)) break;
      ++acc_uses[buf];
      tc_fence_after();
      const uint32_t t_base = tmem + ((uint32_t)(q * 32) << 16) + buf * C::ACC_COLS;
      const int nch = (it.count + 31) >> 5;
      const int seg_row0 = it.seg_off + it.c * BN;
      const int n_glob = it.m * BM + row_in_tile;
      // Columns this CTA finishes: all of them, or with split-K one slice of the tile
      // (dense: every split reduces BN/S columns once all partials exist) or the whole
      // tile in the CTA that completes it (grouped: items may exceed one wave).
      int c_begin = 0, c_end = it.count;
      bool finish = true;
      if (S > 1) {
        float* mine = p.ws + ((size_t)it.tile * S + it.ks) * (size_t)(BN * BM) + row_in_tile;
        for (int ch = 0; ch < nch; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_base + ch * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(mine + (ch * 32 + j) * BM, __uint_as_float(r[j]));
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool parallel = p.chunk_prefix == nullptr;  // host guarantees one wave
        if (q == 0 && lane == 0) {
          __threadfence();
          const int old = atomicAdd(p.tile_sem + it.tile, 1);
          int ok = 1;
          if (parallel) {
            ok = 0;
            for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
              if (sem_acquire(p.tile_sem + it.tile) >= S) { ok = 1; break; }
              if (*abort_flag) break;
              if (i > 16) __nanosleep(32);
            }
            if (!ok) {
              report_error(p.err, kErrMbarTimeout);
              *abort_flag = 1;
            }
          } else {
            ok = old == S - 1;
            if (ok) p.tile_sem[it.tile] = 0;  // every split has arrived: re-arm for the next call
            __threadfence();
          }
          s.fix_last = ok;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        finish = s.fix_last != 0;
        if (parallel) {
          const int width = (BN + S - 1) / S;
          c_begin = it.ks * width;
          c_end = min(it.count, c_begin + width);
        }
      }
      if (finish) {
        const bool valid_n = n_glob < p.n_valid;
        const int nchunks = c_end > c_begin ? (c_end - c_begin + 31) >> 5 : 0;
        for (int ch = 0; ch < nchunks; ++ch) {
          const int col0 = c_begin + ch * 32;
          const int ncols = min(32, c_end - col0);
          float v[32];
          load_cols<BN>(t_base, p, it, S, col0, ncols, row_in_tile, v);
          if (p.epi_mode == kEpiSiluQuant) {
            // Tile rows 0..63 are gate features, 64..127 the matching up features of
            // intermediate columns [64m, 64m+64).  Pair them through shared memory,
            // form silu(g)*u and quantize to MXFP8 (32-feature blocks = one warp).
            if (q >= 2) {
#pragma unroll
              for (int j = 0; j < 32; ++j) s.xch[j][(q - 2) * 32 + lane] = v[j];
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (q < 2) {
              // h = silu(gate) * up for 32 token columns of this lane's feature, written
              // back over the up values this lane read (own column of the padded tile),
              // then read transposed: lane L owns token column L and its 32 consecutive
              // features, so the MXFP8 block maximum needs no shuffles and the row
              // leaves as two 16-byte stores.
#pragma unroll
              for (int j = 0; j < 32; ++j) s.xch[j][q * 32 + lane] = siluf_(v[j]) * s.xch[j][q * 32 + lane];
              __syncwarp();
              if (lane < ncols) {
                float h[32];
                float amax = 0.f;
#pragma unroll
                for (int f = 0; f < 32; ++f) {
                  h[f] = s.xch[lane][q * 32 + f];
                  amax = fmaxf(amax, fabsf(h[f]));
                }
                const uint8_t code = mx_scale_e8m0(amax);
                const float inv = mx_inv_scale(code);
                uint32_t w8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  w8[i] = uint32_t(f32_to_e4m3(h[4 * i] * inv)) | (uint32_t(f32_to_e4m3(h[4 * i + 1] * inv)) << 8) |
                          (uint32_t(f32_to_e4m3(h[4 * i + 2] * inv)) << 16) |
                          (uint32_t(f32_to_e4m3(h[4 * i + 3] * inv)) << 24);
                const int row = seg_row0 + col0 + lane;
                const int feat0 = it.m * 64 + q * 32;  // first intermediate column of the block
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) + (size_t)row * p.ldo + feat0);
                dst[0] = make_uint4(w8[0], w8[1], w8[2], w8[3]);
                dst[1] = make_uint4(w8[4], w8[5], w8[6], w8[7]);
                const int kb = feat0 >> 5;
                uint8_t* sf = p.out_sf + ((size_t)(row >> 7) * (p.ldo >> 7) + (kb >> 2)) * 512;
                sf[sf_atom_offset(row & 127, kb & 3)] = code;
              }
            }
            asm volatile("bar.sync 2, 128;" ::: "memory");
          } else if (p.epi_mode == kEpiArgmaxPartial) {
            // Vocab-tile argmax: reduce each token column over this tile's 128 rows into
            // one packed (orderable logit, ~id) word; the max over words gives the largest
            // logit with the smallest id on ties.
            unsigned long long* part = reinterpret_cast<unsigned long long*>(p.out);
            if (p.row_temp != nullptr && (p.sample_any == nullptr || __ldg(p.sample_any) > 0.f)) {
              // Sampling rows: Gumbel-perturbed scaled logits (same noise on every rank).
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int row = seg_row0 + col0 + j;
                const float t = j < ncols ? __ldg(p.row_temp + row) : 0.f;
                if (t > 0.f)
                  v[j] = v[j] / t + gumbel_noise((unsigned long long)__ldg(p.row_seed + row), __ldg(p.row_pos + row),
                                                 p.id_offset + n_glob);
              }
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              unsigned long long key = valid_n ? pack_argmax(v[j], n_glob) : 0ull;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffff, key, o);
                key = other > key ? other : key;
              }
              if (lane == 0) s.red[q][j] = key;
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (q == 0) {
              const int col = col0 + lane;
              unsigned long long key = s.red[0][lane];
#pragma unroll
              for (int w = 1; w < 4; ++w) key = s.red[w][lane] > key ? s.red[w][lane] : key;
              if (lane < ncols) part[(size_t)(seg_row0 + col) * p.ldo + it.m] = key;
            }
            asm volatile("bar.sync 2, 128;" ::: "memory");
          } else if (p.epi_mode == kEpiScatterScaled) {
            // Destination rows and routing weights: the same address for all lanes, so
            // each is one broadcast load; all 32 are issued before the stores.
            int dst[32];
            float scl[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const bool ok = j < ncols;
              dst[j] = ok ? __ldg(p.row_dst + seg_row0 + col0 + j) : 0;
              scl[j] = ok ? __ldg(p.row_scale + seg_row0 + col0 + j) : 0.f;
            }
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + n_glob;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (valid_n && j < ncols) o[(size_t)dst[j] * p.ldo] = __float2bfloat16_rn(v[j] * scl[j]);
          } else if (p.epi_mode == kEpiPushLL) {
            // Row-parallel partial sums straight into the fused all-reduce's receive slots:
            // lanes 4i..4i+3 hold features 4i..4i+3 of every token column; two shuffles
            // gather them into lane 4i, which stores one LL line per token (8 lanes x 16 B
            // = 128 contiguous bytes per store instruction).
            const uint32_t E = *reinterpret_cast<const volatile uint32_t*>(p.push_epoch) + 1u;
            const int W = p.push_world, L = p.n_valid >> 2;
            const int per = (p.push_rows + W - 1) / W;
            const size_t line = (size_t)(n_glob >> 2);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float nx = __shfl_down_sync(0xffffffff, v[j], 1);
              const uint32_t pk = peer::pack_bf16x2(v[j], nx);
              const uint32_t pk2 = __shfl_down_sync(0xffffffff, pk, 2);
              const int row = seg_row0 + col0 + j;
              if ((lane & 3) == 0 && j < ncols && valid_n) {
                if (p.push_mode == FAR_TWOSHOT) {
                  const int owner = min(row / per, W - 1);
                  peer::st_ll16(static_cast<uint4*>(p.push_part[owner]) +
                                    ((size_t)p.push_rank * per + (row - owner * per)) * L + line, pk, pk2, E);
                } else {
                  const int par = E & 1;
                  for (int q = 0; q < W; ++q)
                    peer::st_ll16(static_cast<uint4*>(p.push_part[q]) +
                                      (((size_t)par * W + p.push_rank) * FAR_ONESHOT_ROWS + row) * L + line,
                                  pk, pk2, E);
                }
              }
            }
          } else if (p.epi_mode == kEpiStoreF32) {
            float* o = reinterpret_cast<float*>(p.out) + it.ks * p.split_stride * split_off +
                       (size_t)(seg_row0 + col0) * p.ldo + n_glob;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (valid_n && j < ncols) o[(size_t)j * p.ldo] = v[j];
          } else {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)(seg_row0 + col0) * p.ldo + n_glob;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (valid_n && j < ncols) o[(size_t)j * p.ldo] = __float2bfloat16_rn(v[j]);
          }
        }
      }
      if (S > 1 && p.chunk_prefix == nullptr) {
        // Second arrival: once all S splits have read every partial, the last re-arms the counter.
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (q == 0 && lane == 0 && atomicAdd(p.tile_sem + it.tile, 1) == 2 * S - 1) atomicExch(p.tile_sem + it.tile, 0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace gemm
}  // namespace zs

// ------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D e4m3 matrix [rows, k] (k contiguous) with a {128 x box_rows} 128B-swizzled box.
int make_tmap_u8(CUtensorMap* m, const void* base, int64_t rows, int64_t k, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k};
  cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Activations [rows, k] viewed as {128 B, rows, k/128 tiles}: one box = box_rows rows of
// kt_box consecutive 128-byte K tiles, laid out in shared memory tile after tile.
int make_tmap_b3(CUtensorMap* m, const void* base, int64_t rows, int64_t k, int box_rows, int kt_box) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(k / 128)};
  cuuint64_t strides[2] = {(cuuint64_t)k, 128};
  cuuint32_t box[3] = {128, (cuuint32_t)box_rows, (cuuint32_t)kt_box};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Pre-tiled weights: [tiles][128 rows][128 B] viewed as a 3-D tensor whose box is one
// whole contiguous tile.
int make_tmap_tiled(CUtensorMap* m, const void* base, int64_t tiles) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[3] = {128, 128, (cuuint64_t)tiles};
  cuuint64_t strides[2] = {128, 128 * 128};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int STAGES, bool FP4>
int launch(const GemmMxf8Args& p, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tbf,
           cudaStream_t stream) {
  using namespace zs::gemm;
  int grid = num_sms();
  if (p.chunk_prefix == nullptr) {
    const int splits = p.k_splits > 1 ? p.k_splits : (p.fix_splits > 1 ? p.fix_splits : 1);
    const int items = ((p.m_rows + BN - 1) / BN) * (p.n_pad / BM) * splits;
    if (items == 0) return 0;
    grid = items < grid ? items : grid;
  } else if (p.max_items > 0 && p.max_items < grid) {
    grid = p.max_items;
  }
  using CF = Cfg<BN, STAGES, FP4>;
  const size_t smem = sizeof(typename CF::Smem) + 1024;
  auto kern = gemm_mxf8_kernel<BN, STAGES, FP4>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  zs_launch(kern, grid, CF::THREADS, smem, stream, ta, tb, tbf, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -15;
}

}  // namespace

extern "C" int zs_gemm_mxf8(const GemmMxf8Args* args, cudaStream_t stream) {
  using namespace zs::gemm;
  const GemmMxf8Args& p = *args;
  if (p.k % BK != 0 || p.n_pad % BM != 0 || p.k <= 0 || p.n_pad <= 0) return -10;
  if ((reinterpret_cast<uintptr_t>(p.a) & 15) || (reinterpret_cast<uintptr_t>(p.b) & 15) ||
      (reinterpret_cast<uintptr_t>(p.sfa) & 15) || (reinterpret_cast<uintptr_t>(p.sfb) & 15))
    return -11;
  if (p.b_rows % BM != 0) return -12;
  // The SiLU epilogue stores 32-byte rows of MXFP8 output.
  if (p.epi_mode == kEpiSiluQuant && ((p.ldo & 15) || (reinterpret_cast<uintptr_t>(p.out) & 15))) return -23;
  if (p.k_splits > 1 && (p.chunk_prefix != nullptr || p.epi_mode != kEpiStoreF32)) return -16;
  if (p.fix_splits > 1) {
    if (p.k_splits > 1 || p.fix_splits > kMaxFixSplits || (p.k / BK) % p.fix_splits != 0 || p.ws == nullptr ||
        p.tile_sem == nullptr)
      return -19;
    const int bn_ = p.block_n == 32 ? 32 : 128;
    const int tiles = ((p.m_rows + bn_ - 1) / bn_) * (p.n_pad / BM);
    if (p.chunk_prefix == nullptr && tiles > p.max_tiles) return -20;
    // Dense split-K waits for the tile's other splits, so every item must be resident at once.
    if (p.chunk_prefix == nullptr && tiles * p.fix_splits > num_sms()) return -21;
  }
  const int bn = p.block_n == 32 ? 32 : 128;
  if (p.epi_mode == kEpiPushLL) {
    // Whole-K items, dense, hidden a multiple of 4, every receive buffer present, rows
    // within the one-shot capacity when pushing to every rank.
    if (p.chunk_prefix != nullptr || p.k_splits > 1 || p.fix_splits > 1 || (p.n_valid & 3) || p.push_epoch == nullptr ||
        p.push_world < 1 || p.push_world > 8 || p.push_rank < 0 || p.push_rank >= p.push_world ||
        p.push_rows != p.m_rows || (p.push_mode != FAR_TWOSHOT && p.push_mode != FAR_ONESHOT) ||
        (p.push_mode == FAR_ONESHOT && p.m_rows > FAR_ONESHOT_ROWS))
      return -24;
    for (int q = 0; q < p.push_world; ++q)
      if (p.push_part[q] == nullptr) return -24;
  }
  if (p.chunk_prefix != nullptr && p.chunk_rows != bn) return -17;
  if (p.last_mt < 0 || p.last_m0 < 0 || (p.last_mt > 0 && (p.chunk_prefix == nullptr || p.last_m0 + p.last_mt > p.n_pad / BM)))
    return -25;
  if (p.chunk_prefix != nullptr && p.groups > kMaxGroups) return -18;
  CUtensorMap ta, tb;
  if (p.a_fp4) {
    // Packed e2m1 tiles (8 KiB each) reach shared memory by plain bulk copies; the map
    // only has to be a valid descriptor of the buffer.
    if (!p.a_tiled) return -22;
    if (make_tmap_tiled(&ta, p.a, (int64_t)p.groups * (p.n_pad / BM) * (p.k / BK) / 2) != 0) return -13;
  } else if (p.a_tiled) {
    if (make_tmap_tiled(&ta, p.a, (int64_t)p.groups * (p.n_pad / BM) * (p.k / BK)) != 0) return -13;
  } else if (make_tmap_u8(&ta, p.a, (int64_t)p.groups * p.n_pad, p.k, BM) != 0) {
    return -13;
  }
  if (make_tmap_u8(&tb, p.b, p.b_rows, p.k, 16) != 0) return -14;
  CUtensorMap tbf;
  if (make_tmap_b3(&tbf, p.b, p.b_rows, p.k, bn, Cfg<32, 4, false>::KT) != 0) return -14;
  if (p.a_fp4) return bn == 32 ? launch<32, 3, true>(p, ta, tb, tbf, stream) : launch<128, 2, true>(p, ta, tb, tbf, stream);
  return bn == 32 ? launch<32, 4, false>(p, ta, tb, tbf, stream) : launch<128, 3, false>(p, ta, tb, tbf, stream);
}

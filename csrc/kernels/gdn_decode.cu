// GatedDeltaNet decode step for sm_100a: persistent, TMA-pipelined state streaming.
//
// A decode step reads and rewrites the fp32 recurrent state of every (token, value
// head): 64 KiB in + 64 KiB out, with almost no math per byte, so the kernel is built
// as a pure streaming pipeline:
//   * one CTA per SM walks a static list of (row, value head) items;
//   * a producer warp stages each item's state (one 64 KiB cp.async.bulk), its conv
//     windows, conv weights and projected q/k/v/z slices into a 3-deep shared-memory
//     ring (mbarrier transaction counts), running up to 3 items ahead;
//   * 16 compute warps (4 threads per value row, 32 state coefficients each) run the
//     causal conv + SiLU, q/k L2 norms, the delta rule and the gated RMSNorm from
//     shared memory, write the new state / windows back in place and emit the output
//     (bf16 and/or one MXFP8 block per 32 values);
//   * the producer writes each finished stage back with bulk stores
//     (cp.async.bulk.global.shared::cta) before reusing it, so loads, compute and
//     stores of different items overlap.
// Conv windows are double-buffered by position parity (the window preceding position p
// lives in buffer p & 1): an item reads buffer p & 1 and writes buffer (p+1) & 1, so
// the value heads sharing a q/k head read the old q/k window while the owner (the
// first value head of the group) writes the new one.
//
// Row groups (TMAX = 4: a speculative verify pass over the last token + K drafts, the
// roll-back replay of the accepted rows): an item is (sequence, value head) with up to 4
// consecutive rows; the state is read once, stepped through the rows in registers and
// written once (to out_slots[seq] when given), each row's output emitted in turn.  The
// q/k windows are left to the follow-up window kernel of the prefill path: with an even
// row count the new window lands in the buffer the other value heads read.
//
// Reference parity: worker/zstep_worker/kernels_sm120/qwen35_ops.py:659-935 (conv,
// delta rule, gated norm; state stored [V, K]) and the fused decode kernels of
// kernels_sm120/csrc/qwen35_ops_kernels.cu:354-757.
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace gdn_dec {

constexpr int DK = 128, DV = 128;
constexpr int STAGES = 3;
constexpr int COMPUTE_WARPS = 16;
constexpr int THREADS = COMPUTE_WARPS * 32 + 32;  // + producer warp
constexpr uint32_t STATE_BYTES = DK * DV * 4;

template <int TMAX>
struct Stage {
  float state[DV * DK];                // [v][k]
  __nv_bfloat16 x[TMAX][3 * 128];      // projected q | k | v channels of each row (conv inputs)
  __nv_bfloat16 z[TMAX][128];          // gate input z of each row
  __nv_bfloat16 win[3 * 128 * 3];      // conv windows (q | k | v), 3 taps per channel
  __nv_bfloat16 w[3 * 128 * 4];        // conv weights (q | k | v), 4 taps per channel
};

template <int TMAX>
struct Smem {
  Stage<TMAX> st[STAGES];
  __nv_bfloat16 conv_out[TMAX][3 * 128];  // q | k | v after conv + SiLU of each row (bf16-rounded values)
  float o[TMAX][DV];                      // delta-rule outputs of each row, before the gated norm
  float red[TMAX][8];                     // per row: sums of squares of q (warps 0-3) and k (4-7)
  float red_o[TMAX][4];                   // per row: sums of squares of o (4 warps)
  float gate[TMAX][2];                    // beta and the decay g of each row of the item
  uint64_t full[STAGES];
  uint64_t computed[STAGES];
  int abort_flag;
};

__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(ssrc)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ bool wait_flag(uint64_t* bar, uint32_t phase, int* err, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
    if (*abort_flag) return false;
    if (i > 32) __nanosleep(32);
  }
  report_error(err, kErrMbarTimeout);
  *abort_flag = 1;
  return false;
}

// An item's rows [row, row + nrows) (nrows 0: nothing to do), value head, q/k head, state
// slot read, slot written, and the position of its first row.
struct ItemInfo {
  int row, nrows, vh, kh, slot, oslot, pos;
};

template <int TMAX>
__device__ __forceinline__ ItemInfo item_info(const GdnArgs& a, int idx) {
  ItemInfo it;
  it.vh = idx % a.num_v_heads;
  it.kh = it.vh / (a.num_v_heads / a.num_k_heads);
  if (TMAX == 1) {
    it.row = idx / a.num_v_heads;
    it.nrows = 1;
    it.slot = it.oslot = a.slots[it.row];
  } else {
    const int seq = idx / a.num_v_heads;
    it.row = a.seq_start[seq];
    it.nrows = a.seq_start[seq + 1] - it.row;
    if (it.nrows > TMAX) it.nrows = 0;  // outside the contract: reported by the producer, skipped
    it.slot = it.nrows > 0 ? a.slots[it.row] : 0;
    it.oslot = a.out_slots != nullptr ? a.out_slots[seq] : it.slot;
  }
  it.pos = it.nrows > 0 ? a.positions[it.row] : 0;
  return it;
}

// Write back a finished stage: state, the new conv windows (q/k only by the first value
// head of the q/k head's group, and only for single-row items), all as bulk stores from
// shared memory.
template <int TMAX>
__device__ __forceinline__ void store_stage(const GdnArgs& a, Stage<TMAX>& st, const ItemInfo& it, int conv_dim) {
  if (it.nrows == 0) return;
  const int ratio = a.num_v_heads / a.num_k_heads;
  float* gstate = a.ssm_state + ((size_t)it.oslot * a.num_v_heads + it.vh) * DV * DK;
  bulk_store(gstate, st.state, STATE_BYTES);
  __nv_bfloat16* cs = static_cast<__nv_bfloat16*>(a.conv_state) +
                      ((size_t)it.oslot * 2 + ((it.pos + it.nrows) & 1)) * conv_dim * 3;
  if (TMAX == 1 && it.vh % ratio == 0) {
    bulk_store(cs + (size_t)it.kh * 128 * 3, st.win, 128 * 3 * 2);
    bulk_store(cs + (size_t)(a.num_k_heads + it.kh) * 128 * 3, st.win + 128 * 3, 128 * 3 * 2);
  }
  bulk_store(cs + (size_t)(2 * a.num_k_heads * 128 + it.vh * 128) * 3, st.win + 2 * 128 * 3, 128 * 3 * 2);
  bulk_commit();
}

template <int TMAX>
__global__ void __launch_bounds__(THREADS, 1) gdn_decode_tma_kernel(const GdnArgs a, int total_items) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  using Sm = Smem<TMAX>;
  Sm& s = *reinterpret_cast<Sm*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hk = a.num_k_heads, Hv = a.num_v_heads;
  const int conv_dim = 2 * Hk * DK + Hv * DV;
  volatile int* abort_flag = &s.abort_flag;
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.computed[i], 1);
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == COMPUTE_WARPS) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      ItemInfo pend[STAGES];
      int n_local = 0;
      const __nv_bfloat16* proj = static_cast<const __nv_bfloat16*>(a.proj);
      const __nv_bfloat16* cw = static_cast<const __nv_bfloat16*>(a.conv_w);
      const __nv_bfloat16* csg = static_cast<const __nv_bfloat16*>(a.conv_state);
      for (int idx = blockIdx.x; idx < total_items && !*abort_flag; idx += gridDim.x, ++n_local) {
        const int sidx = n_local % STAGES;
        Stage<TMAX>& st = s.st[sidx];
        if (n_local >= STAGES) {
          // Stage reuse: write back the item computed STAGES items ago first.
          if (!wait_flag(&s.computed[sidx], ((n_local - STAGES) / STAGES) & 1, a.err, abort_flag)) break;
          store_stage<TMAX>(a, st, pend[sidx], conv_dim);
          bulk_wait_read0();
        }
        const ItemInfo it = item_info<TMAX>(a, idx);
        pend[sidx] = it;
        if (it.nrows == 0) {  // empty sequence (or too many rows: reported): arrive, no copies
          if (TMAX > 1 && a.seq_start[idx / Hv + 1] - a.seq_start[idx / Hv] > TMAX) report_error(a.err, kErrBadShape);
          mbar_expect_tx(&s.full[sidx], 0);
          continue;
        }
        const bool fresh = it.pos == 0;
        const uint32_t bytes =
            (fresh ? 0u : STATE_BYTES + 3 * 128 * 3 * 2) + it.nrows * 4 * 128 * 2 + 3 * 128 * 4 * 2;
        mbar_expect_tx(&s.full[sidx], bytes);
        for (int r = 0; r < it.nrows; ++r) {
          const __nv_bfloat16* prow = proj + (size_t)(it.row + r) * a.ld_proj;
          bulk_load(st.x[r], prow + it.kh * 128, 256, &s.full[sidx]);
          bulk_load(st.x[r] + 128, prow + (Hk + it.kh) * 128, 256, &s.full[sidx]);
          bulk_load(st.x[r] + 256, prow + 2 * Hk * 128 + it.vh * 128, 256, &s.full[sidx]);
          bulk_load(st.z[r], prow + conv_dim + it.vh * 128, 256, &s.full[sidx]);
        }
        bulk_load(st.w, cw + (size_t)it.kh * 128 * 4, 1024, &s.full[sidx]);
        bulk_load(st.w + 512, cw + (size_t)(Hk + it.kh) * 128 * 4, 1024, &s.full[sidx]);
        bulk_load(st.w + 1024, cw + (size_t)(2 * Hk * 128 + it.vh * 128) * 4, 1024, &s.full[sidx]);
        if (!fresh) {
          const __nv_bfloat16* cs = csg + ((size_t)it.slot * 2 + (it.pos & 1)) * conv_dim * 3;
          bulk_load(st.win, cs + (size_t)it.kh * 128 * 3, 768, &s.full[sidx]);
          bulk_load(st.win + 384, cs + (size_t)(Hk + it.kh) * 128 * 3, 768, &s.full[sidx]);
          bulk_load(st.win + 768, cs + (size_t)(2 * Hk * 128 + it.vh * 128) * 3, 768, &s.full[sidx]);
          bulk_load(st.state, a.ssm_state + ((size_t)it.slot * Hv + it.vh) * DV * DK, STATE_BYTES, &s.full[sidx]);
        }
      }
      // Drain: write back the last (up to STAGES) items, then wait for all stores.
      const int first = n_local > STAGES ? n_local - STAGES : 0;
      for (int j = first; j < n_local && !*abort_flag; ++j) {
        const int sidx = j % STAGES;
        if (!wait_flag(&s.computed[sidx], (j / STAGES) & 1, a.err, abort_flag)) break;
        store_stage<TMAX>(a, s.st[sidx], pend[sidx], conv_dim);
      }
      bulk_wait_all0();
      // Loads that were issued but never consumed (abort): wait for them to land.
      for (int j = first; j < n_local; ++j)
        if (!mbar_wait(&s.full[j % STAGES], (j / STAGES) & 1, nullptr)) report_error(a.err, kErrDrainTimeout);
    }
    return;
  }

  // -------------------------------------------------------------------- compute warps
  const int t = threadIdx.x;  // 0..511
  const int vr = t >> 2, kq = t & 3;
  int n_local = 0;
  for (int idx = blockIdx.x; idx < total_items; idx += gridDim.x, ++n_local) {
    const int sidx = n_local % STAGES;
    Stage<TMAX>& st = s.st[sidx];
    if (!wait_flag(&s.full[sidx], (n_local / STAGES) & 1, a.err, abort_flag)) break;
    const ItemInfo it = item_info<TMAX>(a, idx);
    const bool fresh = it.pos == 0;
    // Gates of every row (threads 384.., idle during the conv): their loads and
    // transcendentals overlap the first row's conv instead of sitting on each row's path.
    if (t >= 384 && t < 384 + it.nrows) {
      const int r = t - 384;
      const __nv_bfloat16* prow = static_cast<const __nv_bfloat16*>(a.proj) + (size_t)(it.row + r) * a.ld_proj;
      const int boff = conv_dim + Hv * DV;
      const float b_raw = __bfloat162float(prow[boff + it.vh]);
      const float a_raw = __bfloat162float(prow[boff + Hv + it.vh]);
      const float sp_in = a_raw + a.dt_bias[it.vh];
      const float softplus = sp_in > 20.f ? sp_in : log1pf(__expf(sp_in));
      s.gate[r][0] = sigmoidf_(b_raw);
      s.gate[r][1] = __expf(-__expf(a.a_log[it.vh]) * softplus);
    }
    // State row vr, 32 coefficients per thread, held in registers across the item's rows.
    // The 4 threads of a row own interleaved 16-byte pieces: piece i of thread kq covers
    // k = seg(i)*16 + kq*4 + 0..3 with seg(i) = (i + vr) & 7, so each quarter-warp's
    // 128-bit shared accesses (2 rows x 4 threads) fall in distinct banks.
    float* srow = st.state + vr * DK;
    float c[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k0 = ((i + vr) & 7) * 16 + kq * 4;
      const float4 f = fresh ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<const float4*>(srow + k0);
      c[4 * i] = f.x; c[4 * i + 1] = f.y; c[4 * i + 2] = f.z; c[4 * i + 3] = f.w;
    }
    // 1. conv + SiLU of every row (threads 0..383, one channel each, rows in order: the
    //    window shifts in place).  It does not depend on the state, so all rows go before
    //    the first barrier.
    if (t < 384) {
      __nv_bfloat16* win = st.win + t * 3;
      const __nv_bfloat16* w = st.w + t * 4;
      const float c0 = __bfloat162float(w[0]), c1 = __bfloat162float(w[1]), c2 = __bfloat162float(w[2]),
                  c3 = __bfloat162float(w[3]);
      float w0 = fresh ? 0.f : __bfloat162float(win[0]);  // a fresh sequence's window is all zeros
      float w1 = fresh ? 0.f : __bfloat162float(win[1]);
      float w2 = fresh ? 0.f : __bfloat162float(win[2]);
      for (int r = 0; r < it.nrows; ++r) {
        const float x = __bfloat162float(st.x[r][t]);
        const float acc = c0 * w0 + c1 * w1 + c2 * w2 + c3 * x;
        w0 = w1;
        w1 = w2;
        w2 = x;
        const __nv_bfloat16 yb = __float2bfloat16_rn(siluf_(acc));
        s.conv_out[r][t] = yb;
        const float y = __bfloat162float(yb);
        // Partial sums of squares: warps 0-3 hold q, 4-7 hold k.
        const float sq = warp_sum(y * y);
        if (lane == 0 && warp < 8) s.red[r][warp] = sq;
      }
      if (it.nrows > 0) {
        win[0] = __float2bfloat16_rn(w0);
        win[1] = __float2bfloat16_rn(w1);
        win[2] = __float2bfloat16_rn(w2);
      }
    }
    asm volatile("bar.sync 3, 512;" ::: "memory");  // compute warps only
    // 2. delta rule over the rows, the 32 coefficients of state row vr in registers; the
    //    only exchanges are within the 4 threads of a row (shuffles), so no block barrier.
    for (int r = 0; r < it.nrows; ++r) {
      const float rq = rsqrtf(s.red[r][0] + s.red[r][1] + s.red[r][2] + s.red[r][3] + 1e-6f) * rsqrtf((float)DK);
      const float rk = rsqrtf(s.red[r][4] + s.red[r][5] + s.red[r][6] + s.red[r][7] + 1e-6f);
      const float beta = s.gate[r][0], g = s.gate[r][1];
      float kvm = 0.f, o = 0.f;
      float delta;
      if constexpr (TMAX == 1) {
        // One row: q and k in registers (measured faster for the decode step).
        float qk[32], kk[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k0 = ((i + vr) & 7) * 16 + kq * 4;
          const uint2 qu = *reinterpret_cast<const uint2*>(&s.conv_out[r][k0]);
          const uint2 ku = *reinterpret_cast<const uint2*>(&s.conv_out[r][128 + k0]);
          const float2 qa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qu.x));
          const float2 qb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qu.y));
          const float2 ka = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ku.x));
          const float2 kb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ku.y));
          qk[4 * i] = qa.x; qk[4 * i + 1] = qa.y; qk[4 * i + 2] = qb.x; qk[4 * i + 3] = qb.y;
          kk[4 * i] = ka.x; kk[4 * i + 1] = ka.y; kk[4 * i + 2] = kb.x; kk[4 * i + 3] = kb.y;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          c[i] *= g;
          kvm += c[i] * kk[i];
        }
        kvm *= rk;
        kvm += __shfl_xor_sync(0xffffffff, kvm, 1);
        kvm += __shfl_xor_sync(0xffffffff, kvm, 2);
        delta = (__bfloat162float(s.conv_out[r][256 + vr]) - kvm) * beta * rk;  // folds the k norm into delta
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          c[i] += kk[i] * delta;
          o += c[i] * qk[i];
        }
      } else {
        // Row groups: q and k re-read from shared memory in each of the two passes rather
        // than held in registers (with 17 warps per CTA a thread has 96 registers, and the
        // state row alone takes 32; the register form spills here).
        auto ld4 = [&](int off) -> float4 {
          const uint2 u = *reinterpret_cast<const uint2*>(&s.conv_out[r][off]);
          const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
          const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
          return make_float4(lo.x, lo.y, hi.x, hi.y);
        };
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k0 = ((i + vr) & 7) * 16 + kq * 4;
          const float4 k4 = ld4(128 + k0);
          c[4 * i] *= g; c[4 * i + 1] *= g; c[4 * i + 2] *= g; c[4 * i + 3] *= g;
          kvm += c[4 * i] * k4.x;
          kvm += c[4 * i + 1] * k4.y;
          kvm += c[4 * i + 2] * k4.z;
          kvm += c[4 * i + 3] * k4.w;
        }
        kvm *= rk;
        kvm += __shfl_xor_sync(0xffffffff, kvm, 1);
        kvm += __shfl_xor_sync(0xffffffff, kvm, 2);
        delta = (__bfloat162float(s.conv_out[r][256 + vr]) - kvm) * beta * rk;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k0 = ((i + vr) & 7) * 16 + kq * 4;
          const float4 k4 = ld4(128 + k0);
          const float4 q4 = ld4(k0);
          c[4 * i] += k4.x * delta; c[4 * i + 1] += k4.y * delta;
          c[4 * i + 2] += k4.z * delta; c[4 * i + 3] += k4.w * delta;
          o += c[4 * i] * q4.x;
          o += c[4 * i + 1] * q4.y;
          o += c[4 * i + 2] * q4.z;
          o += c[4 * i + 3] * q4.w;
        }
      }
      o *= rq;
      o += __shfl_xor_sync(0xffffffff, o, 1);
      o += __shfl_xor_sync(0xffffffff, o, 2);
      if (kq == 0) s.o[r][vr] = o;
    }
    // The stepped state back to shared memory for the producer's bulk store.
    if (it.nrows > 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k0 = ((i + vr) & 7) * 16 + kq * 4;
        *reinterpret_cast<float4*>(srow + k0) = make_float4(c[4 * i], c[4 * i + 1], c[4 * i + 2], c[4 * i + 3]);
      }
    }
    asm volatile("bar.sync 3, 512;" ::: "memory");  // every row's o is in shared memory
    // 3. gated RMSNorm + output, all rows at once: warps 4r..4r+3 own row r (one value each).
    {
      const int r = t >> 7, vi = t & 127;
      if (r < it.nrows) {
        const int row = it.row + r;
        const float ov = s.o[r][vi];
        const float ss = warp_sum(ov * ov);
        if (lane == 0) s.red_o[r][warp & 3] = ss;
        asm volatile("bar.sync %0, 128;" ::"r"(4 + r) : "memory");  // the 4 warps of row r
        const float tot = s.red_o[r][0] + s.red_o[r][1] + s.red_o[r][2] + s.red_o[r][3];
        const float rstd = rsqrtf(tot / DV + a.eps);
        const float z = __bfloat162float(st.z[r][vi]);
        const float w = __bfloat162float(static_cast<const __nv_bfloat16*>(a.norm_w)[vi]);
        const float y = __bfloat162float(__float2bfloat16_rn(ov * rstd)) * w * siluf_(z);
        const int width = Hv * DV;
        const int col = it.vh * DV + vi;
        if (a.out_bf16 != nullptr)
          static_cast<__nv_bfloat16*>(a.out_bf16)[(size_t)row * width + col] = __float2bfloat16_rn(y);
        if (a.out_q != nullptr) {
          const float yb = __bfloat162float(__float2bfloat16_rn(y));
          const uint8_t code = mx_scale_e8m0(warp_max(fabsf(yb)));
          a.out_q[(size_t)row * width + col] = f32_to_e4m3(yb * mx_inv_scale(code));
          if (lane == 0) {
            const int kb = col >> 5;
            a.out_sf[((size_t)(row >> 7) * (width >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] =
                code;
          }
        }
      }
    }
    // Make the generic-proxy smem writes (state, windows) visible to the bulk stores.
    fence_proxy_async_shared();
    // 4. hand the stage to the producer for write-back (all compute warps are past
    //    their last read of it once they reach this barrier).
    asm volatile("bar.sync 2, 512;" ::: "memory");
    if (t == 0) mbar_arrive(&s.computed[sidx]);
  }
}

}  // namespace gdn_dec
}  // namespace zs

namespace {

template <int TMAX>
int launch_stream(const GdnArgs& a, int items, cudaStream_t stream) {
  using namespace zs::gdn_dec;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int grid = items < sms ? items : sms;
  const size_t smem = sizeof(Smem<TMAX>) + 128;
  cudaFuncSetAttribute(gdn_decode_tma_kernel<TMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  zs_launch(gdn_decode_tma_kernel<TMAX>, grid, THREADS, smem, stream, a, items);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace

extern "C" int zs_gdn_decode(const GdnArgs* args, cudaStream_t stream) {
  using namespace zs::gdn_dec;
  const GdnArgs& a = *args;
  if (a.head_k != DK || a.head_v != DV || a.num_k_heads <= 0 || a.num_v_heads % a.num_k_heads != 0) return -1;
  if (a.ld_proj % 8 != 0) return -1;  // 16-byte aligned projection rows for the bulk copies
  if (a.rows == 0) return 0;
  return launch_stream<1>(a, a.rows * a.num_v_heads, stream);
}

// Row groups of up to ZS_GDN_ROWS_MAX rows per sequence (seq_start), no checkpoints: the
// streaming kernel over (sequence, value head) items.  The final q/k conv windows are
// written by the caller's follow-up window kernel (zs_gdn_prefill).
extern "C" int zs_gdn_decode_rows(const GdnArgs* args, cudaStream_t stream) {
  using namespace zs::gdn_dec;
  const GdnArgs& a = *args;
  if (a.head_k != DK || a.head_v != DV || a.num_k_heads <= 0 || a.num_v_heads % a.num_k_heads != 0) return -1;
  if (a.ld_proj % 8 != 0 || a.seq_start == nullptr) return -1;
  if (a.num_seqs == 0) return 0;
  return launch_stream<ZS_GDN_ROWS_MAX>(a, a.num_seqs * a.num_v_heads, stream);
}

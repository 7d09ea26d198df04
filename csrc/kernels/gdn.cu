// GatedDeltaNet (Qwen3.5 linear attention) varlen prefill for sm_100a (the decode step
// lives in gdn_decode.cu).
//
// One CTA owns one (sequence, value head) pair and fuses the whole layer body:
//   causal depthwise conv (k=4) + SiLU on the q/k/v channels of that head,
//   L2-normalisation of q and k (q additionally scaled by 1/sqrt(dk)),
//   beta = sigmoid(b), g = exp(-exp(A_log) * softplus(a + dt_bias)),
//   delta-rule update of the fp32 state S[dv, dk]:
//       S = g*S ;  kv = S k ;  S += (beta*(v - kv)) k^T ;  o = S q
//   gated RMSNorm o -> bf16(o * rstd) * w * silu(z), optionally quantized to MXFP8
//   for the out_proj GEMM.
// The state row (128 fp32) of each value channel is split across 4 threads (32
// coefficients each), so a CTA of 512 threads streams the whole 64 KiB state with
// 128-byte contiguous accesses per thread; the state loads are issued first so the
// conv/normalisation prologue overlaps their latency.  Decode is one token per CTA;
// prefill walks the sequence's tokens with the state held in registers and
// snapshots it into checkpoint slots at the requested rows (automatic prefix caching
// of recurrent state).
//
// Reference parity: worker/zstep_worker/kernels_sm120/qwen35_ops.py:659-935 (conv,
// delta rule, gated norm; state stored [V, K]) and the fused CUDA decode/prefill
// kernels in kernels_sm120/csrc/qwen35_ops_kernels.cu:354-1067 (checkpoint save and
// restore per row).
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace gdn {

constexpr int DK = 128;
constexpr int DV = 128;
constexpr int THREADS = 512;  // 128 value rows x 4 k-quarters

struct Smem {
  float q[DK];
  float k[DK];
  float v[DV];
  float o[DV];
  float conv[3 * DK + DV][3];  // running conv window (prefill)
  float red[16];
  float scal[4];
};

__device__ __forceinline__ float bf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

__device__ __forceinline__ float block_sum_512(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) t += red[i];
  return t;
}

// Conv + SiLU for the head's 384 channels of one token, writing q/k/v into smem.
// `win` holds the previous 3 inputs per channel; it is shifted in place.
__device__ __forceinline__ void conv_token(const GdnArgs& a, int row, int kh, int vh, Smem& s,
                                           bool fresh_window) {
  const int t = threadIdx.x;
  if (t < 2 * DK + DV) {
    int ch;  // channel index in the conv space
    if (t < DK) ch = kh * DK + t;                                  // q
    else if (t < 2 * DK) ch = a.num_k_heads * DK + kh * DK + (t - DK);  // k
    else ch = 2 * a.num_k_heads * DK + vh * DV + (t - 2 * DK);       // v
    const __nv_bfloat16* proj = static_cast<const __nv_bfloat16*>(a.proj);
    const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(a.conv_w) + (size_t)ch * 4;
    const float x = bf(proj + (size_t)row * a.ld_proj + ch);
    float* win = s.conv[t];
    if (fresh_window) win[0] = win[1] = win[2] = 0.f;
    float acc = bf(w + 0) * win[0] + bf(w + 1) * win[1] + bf(w + 2) * win[2] + bf(w + 3) * x;
    win[0] = win[1];
    win[1] = win[2];
    // The conv window stores the bf16 input (matching the stored conv state).
    win[2] = x;
    const float y = siluf_(acc);
    // Activation is rounded to bf16 like the reference's conv output buffer.
    const float yb = __bfloat162float(__float2bfloat16_rn(y));
    if (t < DK) s.q[t] = yb;
    else if (t < 2 * DK) s.k[t - DK] = yb;
    else s.v[t - 2 * DK] = yb;
  }
}

// The conv window is double-buffered by position parity: the window that precedes the
// token at position p (inputs p-3..p-1) lives in buffer p & 1.  A decode step reads
// buffer p & 1 and writes buffer (p+1) & 1, so the CTAs of the value heads that share
// a q/k head can all read the old q/k window while one of them writes the new one.
__device__ __forceinline__ void load_window(const GdnArgs& a, int slot, int pos, int kh, int vh, Smem& s) {
  const int t = threadIdx.x;
  if (t < 2 * DK + DV) {
    int ch;
    if (t < DK) ch = kh * DK + t;
    else if (t < 2 * DK) ch = a.num_k_heads * DK + kh * DK + (t - DK);
    else ch = 2 * a.num_k_heads * DK + vh * DV + (t - 2 * DK);
    const int conv_dim = 2 * a.num_k_heads * DK + a.num_v_heads * DV;
    const __nv_bfloat16* cs = static_cast<const __nv_bfloat16*>(a.conv_state) +
                              (((size_t)slot * 2 + (pos & 1)) * conv_dim + ch) * 3;
    s.conv[t][0] = bf(cs + 0);
    s.conv[t][1] = bf(cs + 1);
    s.conv[t][2] = bf(cs + 2);
  }
}

__device__ __forceinline__ void store_window(const GdnArgs& a, int slot, int pos, int kh, int vh,
                                             Smem& s, bool owns_qk) {
  const int t = threadIdx.x;
  if (t < 2 * DK + DV) {
    if (t < 2 * DK && !owns_qk) return;
    int ch;
    if (t < DK) ch = kh * DK + t;
    else if (t < 2 * DK) ch = a.num_k_heads * DK + kh * DK + (t - DK);
    else ch = 2 * a.num_k_heads * DK + vh * DV + (t - 2 * DK);
    const int conv_dim = 2 * a.num_k_heads * DK + a.num_v_heads * DV;
    __nv_bfloat16* cs = static_cast<__nv_bfloat16*>(a.conv_state) +
                        (((size_t)slot * 2 + (pos & 1)) * conv_dim + ch) * 3;
    cs[0] = __float2bfloat16_rn(s.conv[t][0]);
    cs[1] = __float2bfloat16_rn(s.conv[t][1]);
    cs[2] = __float2bfloat16_rn(s.conv[t][2]);
  }
}

// L2-normalise q,k in smem, compute beta / decay for this token.
__device__ __forceinline__ void qk_norm_and_gates(const GdnArgs& a, int row, int vh, Smem& s) {
  const int t = threadIdx.x;
  float qq = 0.f, kk = 0.f;
  if (t < DK) qq = s.q[t] * s.q[t];
  if (t < DK) kk = s.k[t] * s.k[t];
  const float sq = block_sum_512(qq, s.red);
  const float sk = block_sum_512(kk, s.red);
  if (t < DK) {
    s.q[t] = s.q[t] * rsqrtf(sq + 1e-6f) * rsqrtf((float)DK);
    s.k[t] = s.k[t] * rsqrtf(sk + 1e-6f);
  }
  if (t == 0) {
    const __nv_bfloat16* proj = static_cast<const __nv_bfloat16*>(a.proj) + (size_t)row * a.ld_proj;
    const int zoff = 2 * a.num_k_heads * DK + a.num_v_heads * DV;
    const int boff = zoff + a.num_v_heads * DV;
    const int aoff = boff + a.num_v_heads;
    const float b_raw = bf(proj + boff + vh);
    const float a_raw = bf(proj + aoff + vh);
    const float sp_in = a_raw + a.dt_bias[vh];
    const float softplus = sp_in > 20.f ? sp_in : log1pf(__expf(sp_in));
    s.scal[0] = sigmoidf_(b_raw);
    s.scal[1] = __expf(-__expf(a.a_log[vh]) * softplus);
  }
  __syncthreads();
}

// Gated RMSNorm of s.o and output (bf16 and/or MXFP8).  Threads 0..127.
__device__ __forceinline__ void gated_norm_out(const GdnArgs& a, int row, int vh, Smem& s) {
  const int t = threadIdx.x;
  float ov = t < DV ? s.o[t] : 0.f;
  const float ss = block_sum_512(ov * ov, s.red);
  if (t < DV) {
    const float rstd = rsqrtf(ss / DV + a.eps);
    const __nv_bfloat16* proj = static_cast<const __nv_bfloat16*>(a.proj) + (size_t)row * a.ld_proj;
    const int zoff = 2 * a.num_k_heads * DK + a.num_v_heads * DV;
    const float z = bf(proj + zoff + vh * DV + t);
    const float w = bf(static_cast<const __nv_bfloat16*>(a.norm_w) + t);
    const float nrm = __bfloat162float(__float2bfloat16_rn(ov * rstd)) * w;
    const float y = nrm * siluf_(z);
    const int width = a.num_v_heads * DV;
    const int col = vh * DV + t;
    if (a.out_bf16 != nullptr)
      static_cast<__nv_bfloat16*>(a.out_bf16)[(size_t)row * width + col] = __float2bfloat16_rn(y);
    if (a.out_q != nullptr) {
      const float yb = __bfloat162float(__float2bfloat16_rn(y));
      const float amax = warp_max(fabsf(yb));
      const uint8_t code = mx_scale_e8m0(amax);
      a.out_q[(size_t)row * width + col] = f32_to_e4m3(yb * mx_inv_scale(code));
      if ((t & 31) == 0) {
        const int kb = col >> 5;
        a.out_sf[((size_t)(row >> 7) * (width >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] =
            code;
      }
    }
  }
}

// Delta-rule step for the 32 coefficients st[] of value row `vr`, k-quarter `kq`.
__device__ __forceinline__ float delta_step(float (&st)[32], int vr, int kq, const Smem& s) {
  const float beta = s.scal[0];
  const float g = s.scal[1];
  float kv = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    st[i] *= g;
    kv += st[i] * s.k[kq * 32 + i];
  }
  kv += __shfl_xor_sync(0xffffffff, kv, 1);
  kv += __shfl_xor_sync(0xffffffff, kv, 2);
  const float delta = (s.v[vr] - kv) * beta;
  float o = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    st[i] += s.k[kq * 32 + i] * delta;
    o += st[i] * s.q[kq * 32 + i];
  }
  o += __shfl_xor_sync(0xffffffff, o, 1);
  o += __shfl_xor_sync(0xffffffff, o, 2);
  return o;
}

__global__ void __launch_bounds__(THREADS, 1) gdn_prefill_kernel(const GdnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  __shared__ Smem s;
  const int seq = blockIdx.x;
  const int vh = blockIdx.y;
  const int r0 = a.seq_start[seq], r1 = a.seq_start[seq + 1];
  if (r0 >= r1) return;
  const int ratio = a.num_v_heads / a.num_k_heads;
  const int kh = vh / ratio;
  const int t = threadIdx.x;
  const int vr = t >> 2, kq = t & 3;
  const int slot = a.slots[r0];
  const int pos0 = a.positions[r0];
  const bool fresh = pos0 == 0;
  float* sp = a.ssm_state + (((size_t)slot * a.num_v_heads + vh) * DV + vr) * DK + kq * 32;
  float st[32];
  if (!fresh) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 f = reinterpret_cast<const float4*>(sp)[i];
      st[4 * i] = f.x; st[4 * i + 1] = f.y; st[4 * i + 2] = f.z; st[4 * i + 3] = f.w;
    }
    load_window(a, slot, pos0, kh, vh, s);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) st[i] = 0.f;
  }
  __syncthreads();
  int ck = 0;  // next checkpoint index for this sequence
  for (int row = r0; row < r1; ++row) {
    conv_token(a, row, kh, vh, s, fresh && row == r0);
    __syncthreads();
    qk_norm_and_gates(a, row, vh, s);
    const float o = delta_step(st, vr, kq, s);
    if (kq == 0) s.o[vr] = o;
    __syncthreads();
    gated_norm_out(a, row, vh, s);
    // Snapshot state (+ conv window) into checkpoint slots requested at this row.
    while (a.ckpt_rows != nullptr && ck < a.max_ckpt && a.ckpt_rows[seq * a.max_ckpt + ck] == row) {
      const int cslot = a.ckpt_slots[seq * a.max_ckpt + ck];
      float* cp = a.ssm_state + (((size_t)cslot * a.num_v_heads + vh) * DV + vr) * DK + kq * 32;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(cp)[i] = make_float4(st[4 * i], st[4 * i + 1], st[4 * i + 2], st[4 * i + 3]);
      store_window(a, cslot, pos0 + (row - r0) + 1, kh, vh, s, (vh % ratio) == 0);
      ++ck;
    }
    __syncthreads();
  }
  // Final state: back to the input slot, or to out_slots[seq] (speculative verify keeps
  // the pre-step state intact for the roll-back replay).
  const int oslot = a.out_slots != nullptr ? a.out_slots[seq] : slot;
  float* op = a.ssm_state + (((size_t)oslot * a.num_v_heads + vh) * DV + vr) * DK + kq * 32;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    reinterpret_cast<float4*>(op)[i] = make_float4(st[4 * i], st[4 * i + 1], st[4 * i + 2], st[4 * i + 3]);
  // The q/k windows are shared by the value heads of a q/k group and written afterwards by
  // gdn_qk_window_kernel; this CTA stores its own v window only.
  store_window(a, oslot, pos0 + (r1 - r0), kh, vh, s, false);
}

// ------------------------------------------------------------------------------------
// Chunked prefill.  Within a chunk of L <= 64 tokens (cumulative log decay gam_t, state
// S0 at the chunk start) the delta rule unrolls to
//     S_t = exp(gam_t) S0 + sum_{i<=t} exp(gam_t - gam_i) u_i k_i^T
// with pseudo-values u solving the unit lower-triangular system
//     u_t + sum_{i<t} A[t][i] u_i = beta_t (v_t - exp(gam_t) S0 k_t),
//     A[t][i] = beta_t exp(gam_t - gam_i) (k_t . k_i),
// so the chunk's outputs and final state are
//     o_t = exp(gam_t) S0 q_t + sum_{i<=t} exp(gam_t - gam_i) (q_t . k_i) u_i,
//     S_L = exp(gam_L) S0 + sum_i exp(gam_L - gam_i) u_i k_i^T.
// All token-pair terms are dense products over the chunk; only S crosses chunks.  Every
// exponent is a difference gam_t - gam_i <= 0 (decays), so nothing overflows.
// The CTA layout matches the token kernel: one CTA per (sequence, value head), the
// 128 x 128 fp32 state in registers (thread = value row vr, k-quarter kq).  Chunks end
// early at checkpoint rows so snapshots land on chunk boundaries.
// ------------------------------------------------------------------------------------
namespace chunk {

constexpr int C = 64;
constexpr int RS = 148;  // row stride in floats: four 32-float quarters padded to 36, + 4

// Quarter padding keeps the 16-byte accesses of the four k-quarters of one row, and of
// eight consecutive rows at one column, in distinct bank groups.
__device__ __forceinline__ int ix(int t, int d) { return t * RS + (d >> 5) * 36 + (d & 31); }

struct Smem {
  float q[C * RS];   // normalised, scaled q
  float k[C * RS];   // normalised k
  float u[C * RS];   // v -> right-hand side -> pseudo-values
  float o[C * RS];   // outputs before the gated norm
  float A[C][C + 1];
  float P[C][C + 1];
  float gam[C];
  float beta[C];
};

__device__ __forceinline__ float4 ld4(const float* base, int t, int d) {
  return *reinterpret_cast<const float4*>(base + ix(t, d));
}
__device__ __forceinline__ float dot4(const float4& a, const float4& b) {
  return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}

// Sums each of p[0..7] over the warp's 32 lanes with 9 shuffles (three halving exchanges,
// then two butterflies); lane l returns the sum of value (l >> 2) & 7.
__device__ __forceinline__ float reduce8(const float (&p)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? p[i] : p[i + 4];
    const float keep = b4 ? p[i + 4] : p[i];
    q[i] = keep + __shfl_xor_sync(0xffffffff, send, 16);
  }
  float z[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? q[i] : q[i + 2];
    const float keep = b3 ? q[i + 2] : q[i];
    z[i] = keep + __shfl_xor_sync(0xffffffff, send, 8);
  }
  float y = (b2 ? z[1] : z[0]) + __shfl_xor_sync(0xffffffff, b2 ? z[0] : z[1], 4);
  y += __shfl_xor_sync(0xffffffff, y, 1);
  y += __shfl_xor_sync(0xffffffff, y, 2);
  return y;
}

__global__ void __launch_bounds__(THREADS, 1) gdn_prefill_chunk_kernel(const GdnArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  const int seq = blockIdx.x;
  const int vh = blockIdx.y;
  const int r0 = a.seq_start[seq], r1 = a.seq_start[seq + 1];
  if (r0 >= r1) return;
  const int ratio = a.num_v_heads / a.num_k_heads;
  const int kh = vh / ratio;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  // Triangular solve and intra-chunk outputs: column vr, i-residue kq.  State products:
  // warp w owns value rows 8w..8w+7 (the same rows as its vr columns), lane owns k
  // columns 4*lane..4*lane+3, so one 16-byte load of a k or q row feeds 32 FMAs.
  const int vr = t >> 2, kq = t & 3;
  const int row0 = warp * 8;
  const int slot = a.slots[r0];
  const int pos0 = a.positions[r0];
  const bool fresh = pos0 == 0;
  const __nv_bfloat16* proj = static_cast<const __nv_bfloat16*>(a.proj);
  const int conv_dim = 2 * a.num_k_heads * DK + a.num_v_heads * DV;
  const int zoff = 2 * a.num_k_heads * DK + a.num_v_heads * DV;
  const int boff = zoff + a.num_v_heads * DV;
  const int aoff = boff + a.num_v_heads;

  float st[32];  // st[4r + c] = S[row0 + r][4 lane + c]
  if (!fresh) {
    const float* sp = a.ssm_state + ((size_t)slot * a.num_v_heads + vh) * DV * DK;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const float4 f = *reinterpret_cast<const float4*>(sp + (size_t)(row0 + r) * DK + lane * 4);
      st[4 * r] = f.x; st[4 * r + 1] = f.y; st[4 * r + 2] = f.z; st[4 * r + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) st[i] = 0.f;
  }
  // Conv channel of threads 0..383 (q | k | v of this head), window in registers.
  int ch = 0;
  float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f, win0 = 0.f, win1 = 0.f, win2 = 0.f;
  if (t < 2 * DK + DV) {
    if (t < DK) ch = kh * DK + t;
    else if (t < 2 * DK) ch = a.num_k_heads * DK + kh * DK + (t - DK);
    else ch = 2 * a.num_k_heads * DK + vh * DV + (t - 2 * DK);
    const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(a.conv_w) + (size_t)ch * 4;
    w0 = bf(w); w1 = bf(w + 1); w2 = bf(w + 2); w3 = bf(w + 3);
    if (!fresh) {
      const __nv_bfloat16* cs = static_cast<const __nv_bfloat16*>(a.conv_state) +
                                (((size_t)slot * 2 + (pos0 & 1)) * conv_dim + ch) * 3;
      win0 = bf(cs); win1 = bf(cs + 1); win2 = bf(cs + 2);
    }
  }
  const float decay_rate = -__expf(a.a_log[vh]);
  const float dtb = a.dt_bias[vh];
  const bool owns_qk = (vh % ratio) == 0;
  auto store_win = [&](int dst_slot, int pos, bool with_qk) {
    if (t < 2 * DK + DV && (t >= 2 * DK || with_qk)) {
      __nv_bfloat16* cs = static_cast<__nv_bfloat16*>(a.conv_state) +
                          (((size_t)dst_slot * 2 + (pos & 1)) * conv_dim + ch) * 3;
      cs[0] = __float2bfloat16_rn(win0);
      cs[1] = __float2bfloat16_rn(win1);
      cs[2] = __float2bfloat16_rn(win2);
    }
  };
  auto store_state = [&](int dst_slot) {
    float* op = a.ssm_state + ((size_t)dst_slot * a.num_v_heads + vh) * DV * DK;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      *reinterpret_cast<float4*>(op + (size_t)(row0 + r) * DK + lane * 4) =
          make_float4(st[4 * r], st[4 * r + 1], st[4 * r + 2], st[4 * r + 3]);
  };

  int ck = 0;
  for (int c0 = r0; c0 < r1;) {
    int c1 = min(r1, c0 + C);
    if (a.ckpt_rows != nullptr && ck < a.max_ckpt) {
      const int cr = a.ckpt_rows[seq * a.max_ckpt + ck];
      if (cr >= c0 && cr < c1 - 1) c1 = cr + 1;
    }
    const int L = c1 - c0;

    // 1. conv + SiLU per channel (bf16-rounded like the token kernel); gates per token
    if (t < 2 * DK + DV) {
      float* dst = t < DK ? s.q : (t < 2 * DK ? s.k : s.u);
      const int d = t & (DK - 1);
      const __nv_bfloat16* src = proj + (size_t)c0 * a.ld_proj + ch;
      for (int j0 = 0; j0 < C; j0 += 16) {
        float xs[16];  // 16 independent loads in flight before the sequential window update
#pragma unroll
        for (int u = 0; u < 16; ++u) xs[u] = j0 + u < L ? bf(src + (size_t)(j0 + u) * a.ld_proj) : 0.f;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          float yb = 0.f;
          if (j0 + u < L) {
            const float x = xs[u];
            const float acc = w0 * win0 + w1 * win1 + w2 * win2 + w3 * x;
            win0 = win1;
            win1 = win2;
            win2 = x;
            yb = __bfloat162float(__float2bfloat16_rn(siluf_(acc)));
          }
          dst[ix(j0 + u, d)] = yb;
        }
      }
    } else if (t < 2 * DK + DV + C) {
      const int j = t - (2 * DK + DV);
      float beta = 0.f, lg = 0.f;
      if (j < L) {
        const __nv_bfloat16* pr = proj + (size_t)(c0 + j) * a.ld_proj;
        const float sp_in = bf(pr + aoff + vh) + dtb;
        const float softplus = sp_in > 20.f ? sp_in : log1pf(__expf(sp_in));
        beta = sigmoidf_(bf(pr + boff + vh));
        lg = decay_rate * softplus;
      }
      s.beta[j] = beta;
      s.gam[j] = lg;
    }
    __syncthreads();

    // 2. cumulative log decay (warp 0), L2 norms of q and k (a warp per token)
    if (warp == 0) {
      float v0 = s.gam[lane], v1 = s.gam[lane + 32];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n0 = __shfl_up_sync(0xffffffff, v0, o);
        const float n1 = __shfl_up_sync(0xffffffff, v1, o);
        if (lane >= o) { v0 += n0; v1 += n1; }
      }
      v1 += __shfl_sync(0xffffffff, v0, 31);
      s.gam[lane] = v0;
      s.gam[lane + 32] = v1;
    }
    for (int j = warp; j < C; j += THREADS / 32) {
      float4 qv = ld4(s.q, j, lane * 4), kv = ld4(s.k, j, lane * 4);
      const float sq = warp_sum(dot4(qv, qv));
      const float sk = warp_sum(dot4(kv, kv));
      const float fq = rsqrtf(sq + 1e-6f) * rsqrtf((float)DK), fk = rsqrtf(sk + 1e-6f);
      qv.x *= fq; qv.y *= fq; qv.z *= fq; qv.w *= fq;
      kv.x *= fk; kv.y *= fk; kv.z *= fk; kv.w *= fk;
      *reinterpret_cast<float4*>(s.q + ix(j, lane * 4)) = qv;
      *reinterpret_cast<float4*>(s.k + ix(j, lane * 4)) = kv;
    }
    __syncthreads();

    // 3. A (strictly lower) and P (lower incl. diagonal) on 4 x 4 tiles of the lower
    //    triangle: 136 tiles, two adjacent lanes per tile splitting the 128 dims.  Only
    //    entries with i < t (A) and i <= t (P) are read later.  Warps 0-8 take the tiles;
    //    the rest go straight on to step 4.
    if (t < 288) {
      const int x = t >> 1, half = t & 1;
      const bool live = x < 136;
      int bi = (int)((sqrtf(8.f * x + 1.f) - 1.f) * 0.5f);
      while ((bi + 1) * (bi + 2) / 2 <= x) ++bi;
      while (bi > 0 && bi * (bi + 1) / 2 > x) --bi;
      const int bj = x - bi * (bi + 1) / 2;
      const int ti0 = bi * 4, ii0 = bj * 4;
      float kk[4][4], qk[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) kk[i][j] = qk[i][j] = 0.f;
      if (live) {
        for (int d = half * 64; d < half * 64 + 64; d += 4) {
          float4 ki[4];
#pragma unroll
          for (int b = 0; b < 4; ++b) ki[b] = ld4(s.k, ii0 + b, d);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float4 kt = ld4(s.k, ti0 + r, d), qt = ld4(s.q, ti0 + r, d);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              kk[r][b] += dot4(kt, ki[b]);
              qk[r][b] += dot4(qt, ki[b]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          kk[r][b] += __shfl_xor_sync(0xffffffff, kk[r][b], 1);
          qk[r][b] += __shfl_xor_sync(0xffffffff, qk[r][b], 1);
        }
      if (live) {
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int ti = ti0 + r, ii = ii0 + b;
            const float dec = ii <= ti ? __expf(s.gam[ti] - s.gam[ii]) : 0.f;
            if (half == 0) s.A[ti][ii] = ii < ti ? s.beta[ti] * dec * kk[r][b] : 0.f;
            else s.P[ti][ii] = dec * qk[r][b];
          }
      }
    }
    // 4. through S0: right-hand side u_j = beta_j (v_j - exp(gam_j) S0 k_j) and the
    //    inter-chunk output term o_j = exp(gam_j) S0 q_j (rows of this warp only)
    for (int j = 0; j < L; ++j) {
      const float4 kv = ld4(s.k, j, lane * 4);
      const float4 qv = ld4(s.q, j, lane * 4);
      float pk[8], pq[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        pk[r] = st[4 * r] * kv.x + st[4 * r + 1] * kv.y + st[4 * r + 2] * kv.z + st[4 * r + 3] * kv.w;
        pq[r] = st[4 * r] * qv.x + st[4 * r + 1] * qv.y + st[4 * r + 2] * qv.z + st[4 * r + 3] * qv.w;
      }
      const float xk = reduce8(pk, lane);
      const float xq = reduce8(pq, lane);
      if ((lane & 3) == 0) {
        const int v = row0 + ((lane >> 2) & 7);
        const float e = __expf(s.gam[j]);
        float* u = s.u + ix(j, v);
        *u = s.beta[j] * (*u - e * xk);
        s.o[ix(j, v)] = e * xq;
      }
    }
    __syncthreads();

    // 5. forward substitution per value column: the four lanes of column vr split the
    //    i-sum (i = kq mod 4) and meet through shuffles, so no block barrier is needed
    for (int j = 1; j < L; ++j) {
      float acc = 0.f;
      for (int i = kq; i < j; i += 4) acc += s.A[j][i] * s.u[ix(i, vr)];
      acc += __shfl_xor_sync(0xffffffff, acc, 1);
      acc += __shfl_xor_sync(0xffffffff, acc, 2);
      if (kq == 0) s.u[ix(j, vr)] -= acc;
      __syncwarp();
    }
    __syncwarp();

    // 6. intra-chunk output term (rows j = kq mod 4 of column vr)
    for (int j = kq; j < L; j += 4) {
      float o = s.o[ix(j, vr)];
      for (int i = 0; i <= j; ++i) o += s.P[j][i] * s.u[ix(i, vr)];
      s.o[ix(j, vr)] = o;
    }
    // 7. carry the state to the chunk end (own 32 coefficients)
    {
      const float gl = s.gam[L - 1];
      const float dl = __expf(gl);
#pragma unroll
      for (int i = 0; i < 32; ++i) st[i] *= dl;
      for (int j = 0; j < L; ++j) {
        const float e = __expf(gl - s.gam[j]);
        const float4 kv = ld4(s.k, j, lane * 4);
        const float4 u0 = ld4(s.u, j, row0), u1 = ld4(s.u, j, row0 + 4);
        const float uw[8] = {u0.x * e, u0.y * e, u0.z * e, u0.w * e, u1.x * e, u1.y * e, u1.z * e, u1.w * e};
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          st[4 * r] += uw[r] * kv.x;
          st[4 * r + 1] += uw[r] * kv.y;
          st[4 * r + 2] += uw[r] * kv.z;
          st[4 * r + 3] += uw[r] * kv.w;
        }
      }
    }
    __syncthreads();

    // 8. gated RMSNorm + output, a warp per token (lane = 4 consecutive columns)
    const int width = a.num_v_heads * DV;
    float zg[C / (THREADS / 32)][4];  // gate inputs of this warp's tokens, loaded together
#pragma unroll
    for (int u = 0; u < C / (THREADS / 32); ++u) {
      const int j = warp + u * (THREADS / 32);
      const __nv_bfloat16* pr = proj + (size_t)(c0 + j) * a.ld_proj + zoff + vh * DV + lane * 4;
#pragma unroll
      for (int e = 0; e < 4; ++e) zg[u][e] = j < L ? bf(pr + e) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < C / (THREADS / 32); ++u) {
      const int j = warp + u * (THREADS / 32);
      if (j >= L) break;
      const int row = c0 + j;
      const int d = lane * 4;
      const float4 ov = ld4(s.o, j, d);
      const float ss = warp_sum(dot4(ov, ov));
      const float rstd = rsqrtf(ss / DV + a.eps);
      const __nv_bfloat16* nw = static_cast<const __nv_bfloat16*>(a.norm_w) + d;
      const float of[4] = {ov.x, ov.y, ov.z, ov.w};
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float nrm = __bfloat162float(__float2bfloat16_rn(of[e] * rstd)) * bf(nw + e);
        y[e] = nrm * siluf_(zg[u][e]);
      }
      const int col = vh * DV + d;
      if (a.out_bf16 != nullptr) {
        __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(a.out_bf16) + (size_t)row * width + col;
        __nv_bfloat162 lo = __floats2bfloat162_rn(y[0], y[1]), hi = __floats2bfloat162_rn(y[2], y[3]);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(ob) = pk;
      }
      if (a.out_q != nullptr) {
        float yb[4], amax = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          yb[e] = __bfloat162float(__float2bfloat16_rn(y[e]));
          amax = fmaxf(amax, fabsf(yb[e]));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 4));  // 8 lanes = one 32-column block
        const uint8_t code = mx_scale_e8m0(amax);
        const float inv = mx_inv_scale(code);
        const uint32_t qw = uint32_t(f32_to_e4m3(yb[0] * inv)) | (uint32_t(f32_to_e4m3(yb[1] * inv)) << 8) |
                            (uint32_t(f32_to_e4m3(yb[2] * inv)) << 16) | (uint32_t(f32_to_e4m3(yb[3] * inv)) << 24);
        *reinterpret_cast<uint32_t*>(a.out_q + (size_t)row * width + col) = qw;
        if ((lane & 7) == 0) {
          const int kb = col >> 5;
          a.out_sf[((size_t)(row >> 7) * (width >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] = code;
        }
      }
    }
    // 9. checkpoints requested at the chunk's last row
    while (a.ckpt_rows != nullptr && ck < a.max_ckpt && a.ckpt_rows[seq * a.max_ckpt + ck] == c1 - 1) {
      const int cslot = a.ckpt_slots[seq * a.max_ckpt + ck];
      store_state(cslot);
      store_win(cslot, pos0 + (c1 - r0), owns_qk);
      ++ck;
    }
    c0 = c1;
    __syncthreads();  // shared tiles are rewritten by the next chunk
  }
  const int oslot = a.out_slots != nullptr ? a.out_slots[seq] : slot;
  store_state(oslot);
  store_win(oslot, pos0 + (r1 - r0), false);  // q/k windows: gdn_qk_window_kernel
}

}  // namespace chunk

// ------------------------------------------------------------------------------------
// Final q/k conv windows, one thread per q/k channel of each (sequence, q/k head).
// Every value-head CTA of a q/k group reads the group's q/k window when it starts, and the
// window after T new rows goes to parity buffer (pos0 + T) & 1: for even T that is the
// buffer being read, and the grid orders sequences fastest, so a value head scheduled a
// wave after its group's first one would read an already advanced window.  The prefill
// kernels therefore store only their own v windows (checkpoint slots excepted: nothing
// reads them during the call) and this kernel, stream-ordered after them, writes the
// last three conv inputs of (old window, new rows) of each q/k channel.
__global__ void gdn_qk_window_kernel(const GdnArgs a) {
  pdl_wait();  // the prefill kernel (every reader of the old windows) has finished
  pdl_trigger();
  const int seq = blockIdx.x, kh = blockIdx.y, t = threadIdx.x;
  const int r0 = a.seq_start[seq], r1 = a.seq_start[seq + 1];
  if (r0 >= r1 || t >= 2 * DK) return;
  const int Hk = a.num_k_heads;
  const int conv_dim = 2 * Hk * DK + a.num_v_heads * DV;
  const int ch = t < DK ? kh * DK + t : Hk * DK + kh * DK + (t - DK);
  const int slot = a.slots[r0], pos0 = a.positions[r0];
  const int oslot = a.out_slots != nullptr ? a.out_slots[seq] : slot;
  const int T = r1 - r0;
  const __nv_bfloat16* proj = static_cast<const __nv_bfloat16*>(a.proj);
  const __nv_bfloat16* old_w = static_cast<const __nv_bfloat16*>(a.conv_state) +
                               (((size_t)slot * 2 + (pos0 & 1)) * conv_dim + ch) * 3;
  __nv_bfloat16 w[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int src = T - 3 + i;  // new row index; negative: entry 3 + src of the old window
    w[i] = src >= 0 ? proj[(size_t)(r0 + src) * a.ld_proj + ch]
                    : (pos0 == 0 ? __float2bfloat16_rn(0.f) : old_w[3 + src]);
  }
  // All three old entries are in registers before the store (it may overwrite them).
  __nv_bfloat16* new_w = static_cast<__nv_bfloat16*>(a.conv_state) +
                         (((size_t)oslot * 2 + ((pos0 + T) & 1)) * conv_dim + ch) * 3;
  new_w[0] = w[0];
  new_w[1] = w[1];
  new_w[2] = w[2];
}

}  // namespace gdn
}  // namespace zs

extern "C" int zs_gdn_prefill(const GdnArgs* args, cudaStream_t stream) {
  const GdnArgs& a = *args;
  if (a.head_k != zs::gdn::DK || a.head_v != zs::gdn::DV || a.num_k_heads <= 0 ||
      a.num_v_heads % a.num_k_heads != 0 || a.seq_start == nullptr)
    return -1;
  if (a.num_seqs == 0) return 0;
  dim3 grid(a.num_seqs, a.num_v_heads);
  const bool chunked = a.impl == 2 || (a.impl == 0 && a.rows >= 16 * a.num_seqs);
  const bool short_rows = a.impl == 0 && a.max_seq_rows >= 1 && a.max_seq_rows <= ZS_GDN_ROWS_MAX &&
                          (a.ckpt_rows == nullptr || a.max_ckpt == 0);
  if (short_rows) {
    // A few rows per sequence (speculative verify / replay): the streaming decode kernel
    // reads and writes each state once.
    const int rc = zs_gdn_decode_rows(&a, stream);
    if (rc != 0) return rc;
  } else if (chunked) {
    const int smem = (int)sizeof(zs::gdn::chunk::Smem);
    static bool attr_set[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 16 && !attr_set[dev]) {
      if (cudaFuncSetAttribute(zs::gdn::chunk::gdn_prefill_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess)
        return -2;
      attr_set[dev] = true;
    }
    zs_launch(zs::gdn::chunk::gdn_prefill_chunk_kernel, grid, zs::gdn::THREADS, smem, stream, a);
  } else {
    zs_launch(zs::gdn::gdn_prefill_kernel, grid, zs::gdn::THREADS, 0, stream, a);
  }
  zs_launch(zs::gdn::gdn_qk_window_kernel, dim3(a.num_seqs, a.num_k_heads), 2 * zs::gdn::DK, 0, stream, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

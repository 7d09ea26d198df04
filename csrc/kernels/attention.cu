// Gated GQA attention over a paged KV cache (Qwen3.5 full-attention layers).
//
//  * prologue: per row, zero-centered RMSNorm of every q and k head ((1 + w) scale),
//    partial rotary embedding (rotate-half over the first `rotary_dim` dims, cos/sin
//    rounded to bf16 as a bf16 rotary cache would be), sigmoid-gate passthrough, and
//    the K/V write into the row's page slot.
//  * split-KV decode: one CTA per (row, kv head, split); one warp per query head of
//    the GQA group; each warp splits into 4 lane groups that stream disjoint tokens
//    (8 lanes x 32 dims per token), with an online softmax per lane group.  Partial
//    (o, m, l) go to scratch and a combine kernel merges the splits, applies the
//    sigmoid gate and emits bf16 and/or MXFP8 for the o_proj GEMM.
//  * varlen prefill reuses the same kernels with each query row's causal context
//    length (position + 1): K/V of the whole chunk are written first, then every
//    query attends over its own prefix.
//
// Reference parity: worker/zstep_worker/kernels_sm120/qwen35_ops.py:187-560 (attention
// prologue, split-K(16) paged GQA decode + gated reduce, varlen gated prefill).
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace attn {

constexpr int D = 256;  // head_dim supported by these kernels

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One CTA per row; one warp per head (q heads then k heads); lane owns 8 dims.
__global__ void prologue_kernel(const AttnArgs a) {
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nh = a.num_q_heads + a.num_kv_heads;
  const int pos = a.positions[row];
  const int half = a.rotary_dim / 2;
  const __nv_bfloat16* qkv = static_cast<const __nv_bfloat16*>(a.qkv) + (size_t)row * a.ld_qkv;
  for (int h = warp; h < nh + a.num_kv_heads; h += blockDim.x >> 5) {
    if (h >= nh) {
      // V head: straight copy into the cache.
      const int kvh = h - nh;
      const int slot = a.slots[row];
      const int page = a.page_table[(size_t)slot * a.max_pages + pos / a.page_size];
      const size_t dst = (((size_t)page * a.page_size + pos % a.page_size) * a.num_kv_heads + kvh) * D;
      const uint4* src = reinterpret_cast<const uint4*>(qkv + a.num_q_heads * 2 * D + a.num_kv_heads * D + kvh * D);
      reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.v_cache) + dst)[lane] = src[lane];
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
      const int slot = a.slots[row];
      const int page = a.page_table[(size_t)slot * a.max_pages + pos / a.page_size];
      const size_t dst = (((size_t)page * a.page_size + pos % a.page_size) * a.num_kv_heads + kvh) * D;
      reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.k_cache) + dst)[lane] = pv;
    }
  }
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 v = __bfloat1622float2(h[j]);
    f[2 * j] = v.x;
    f[2 * j + 1] = v.y;
  }
}

// Partial record per (row, q head, split): o[256] (unnormalised), m, l, 2 pad floats.
constexpr int PREC = D + 4;  // padded to keep each record 16-byte aligned

__global__ void decode_partial_kernel(const AttnArgs a) {
  const int row = blockIdx.x;
  const int kvh = blockIdx.y;
  const int split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = a.num_q_heads / a.num_kv_heads;
  const int qh = kvh * group + warp;
  const int grp = lane >> 3, li = lane & 7;
  const int ctx = a.seq_lens[row];
  const int slot = a.slots[row];
  // Token range of this split, in whole pages.
  const int pages = (ctx + a.page_size - 1) / a.page_size;
  const int pps = (pages + a.num_splits - 1) / a.num_splits;
  const int t_begin = split * pps * a.page_size;
  const int t_end = min(ctx, (split + 1) * pps * a.page_size);

  const float qscale = a.sm_scale * 1.4426950408889634f;  // exp2 domain
  float q[32];
  {
    const __nv_bfloat16* qp = static_cast<const __nv_bfloat16*>(a.q_out) + ((size_t)row * a.num_q_heads + qh) * D + li * 32;
#pragma unroll
    for (int c = 0; c < 4; ++c) load8(qp + c * 8, q + c * 8);
#pragma unroll
    for (int j = 0; j < 32; ++j) q[j] *= qscale;
  }
  float o[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j] = 0.f;
  float m = -INFINITY, l = 0.f;
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(a.k_cache);
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(a.v_cache);
  const int* pt = a.page_table + (size_t)slot * a.max_pages;
  // Every lane runs the same trip count (shuffles need the full warp); a lane group
  // whose token is past the end contributes nothing.
  for (int t0 = t_begin; t0 < t_end; t0 += 4) {
    const int t = t0 + grp;
    const bool valid = t < t_end;
    const int tt = valid ? t : t_begin;
    const int page = __ldg(pt + tt / a.page_size);
    const size_t base = (((size_t)page * a.page_size + tt % a.page_size) * a.num_kv_heads + kvh) * D + li * 32;
    float kf[32];
#pragma unroll
    for (int c = 0; c < 4; ++c) load8(kc + base + c * 8, kf + c * 8);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) s += q[j] * kf[j];
    s += __shfl_xor_sync(0xffffffff, s, 1);
    s += __shfl_xor_sync(0xffffffff, s, 2);
    s += __shfl_xor_sync(0xffffffff, s, 4);
    if (!valid) continue;
    float vf[32];
#pragma unroll
    for (int c = 0; c < 4; ++c) load8(vc + base + c * 8, vf + c * 8);
    if (s > m) {
      const float sc = exp2f(m - s);
      l *= sc;
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] *= sc;
      m = s;
    }
    const float p = exp2f(s - m);
    l += p;
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] += p * vf[j];
  }
  // Merge the 4 lane groups (xor 8, xor 16 swap groups with equal li).
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
    for (int c = 0; c < 8; ++c)
      reinterpret_cast<float4*>(rec + li * 32)[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
    if (li == 0) {
      rec[D] = m;
      rec[D + 1] = l;
    }
  }
}

// One CTA (256 threads, thread = dim) per (row, q head): merge splits, normalise,
// apply sigmoid(gate), write bf16 and/or MXFP8.
__global__ void decode_combine_kernel(const AttnArgs a) {
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
  zs::attn::prologue_kernel<<<a.rows, 256, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

extern "C" int zs_attn_decode(const AttnArgs* args, cudaStream_t stream) {
  const AttnArgs& a = *args;
  if (a.head_dim != zs::attn::D || a.num_kv_heads <= 0 || a.num_q_heads % a.num_kv_heads != 0) return -1;
  const int group = a.num_q_heads / a.num_kv_heads;
  if (group > 32 || a.num_splits < 1 || a.partial == nullptr) return -1;
  if (a.rows == 0) return 0;
  dim3 g1(a.rows, a.num_kv_heads, a.num_splits);
  zs::attn::decode_partial_kernel<<<g1, group * 32, 0, stream>>>(a);
  dim3 g2(a.rows, a.num_q_heads);
  zs::attn::decode_combine_kernel<<<g2, zs::attn::D, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Varlen prefill: identical math with per-row causal context lengths (seq_lens must
// hold position + 1 for every row); the caller runs the prologue for all rows first.
extern "C" int zs_attn_prefill(const AttnArgs* args, cudaStream_t stream) {
  return zs_attn_decode(args, stream);
}

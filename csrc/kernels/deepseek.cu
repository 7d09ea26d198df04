// DeepSeek-style layer kernels: manifold-constrained hyper-connections (mHC), the MLA
// prologue / absorbed attention / value up-projection, the DSA lightning indexer and its
// deterministic top-k, and the MoE combine.
//
// Layouts
//   mHC residual streams X: fp32 [rows, n, H] (n = 4).  Mixing logits of one site:
//   [pre n | post n | res n*n]; partial sums per (row, column slice): [M | sum of squares].
//   Latent KV cache (per layer): bf16 [pages, page_size, kv_lora + rope] rows (c_kv | k_pe).
//   Index key cache (per layer): bf16 [pages, page_size, index_dim].
//   Absorbed weights: W_UK [heads, nope, kv_lora] (latent contiguous), W_UV^T [heads,
//   kv_lora, v] (value dim contiguous), both bf16.
//
// The reference serves this model family through vLLM (worker/zstep_worker/models/
// deepseek_v41.py) and its own mHC kernels (csrc/shm_allreduce.cu:2573 post + collapse +
// RMSNorm, :2687 Sinkhorn statistics); the math here follows the model definition that
// zstep_b200/models/deepseek_ref.py states in fp32.
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace ds {

constexpr int kHcN = 4;                        // residual streams
constexpr int kHcM = 2 * kHcN + kHcN * kHcN;   // mixing logits of one site
constexpr int kPartTok = 4;                    // rows per CTA of the partial kernel
constexpr int kPartCols = 512;                 // columns per CTA of the partial kernel

ZS_DEVICE float bfr(float x) { return __bfloat162float(__float2bfloat16(x)); }

ZS_DEVICE float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

ZS_DEVICE void rope_cs(int pos, int i, int dim, float theta, float& c, float& s) {
  const float inv_freq = powf(theta, -2.0f * i / dim);
  sincosf((float)pos * inv_freq, &s, &c);
  c = bfr(c);
  s = bfr(s);
}

// Quantize 8 consecutive values of one row (columns col..col+7) to MXFP8.  Four
// consecutive lanes hold one 32-element block: they exchange their maxima.
ZS_DEVICE void quant8_store(const float (&v)[8], bool active, int row, int col, int width, uint8_t* q,
                            uint8_t* sf) {
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, 2));
  if (!active) return;
  const uint8_t code = mx_scale_e8m0(amax);
  const float inv = mx_inv_scale(code);
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    w0 |= (uint32_t)f32_to_e4m3(v[j] * inv) << (8 * j);
    w1 |= (uint32_t)f32_to_e4m3(v[4 + j] * inv) << (8 * j);
  }
  *reinterpret_cast<uint2*>(q + (size_t)row * width + col) = make_uint2(w0, w1);
  if ((col & 31) == 0) {
    const int kb = col >> 5;
    sf[((size_t)(row >> 7) * (width >> 7) + (kb >> 2)) * 512 + sf_atom_offset(row & 127, kb & 3)] = code;
  }
}

// ------------------------------------------------------------------------------ mHC
// Partial mixing sums of one site for kPartTok rows x kPartCols columns of every stream.
// mode 0: X as is; mode 1: first X <- res @ X + post * bf16(y) (the previous site's
// update, written back); mode 2: X <- bf16(embed[ids]) in every stream (written).
template <int M>
__global__ void __launch_bounds__(256)
mhc_partial_kernel(MhcPartialArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int t0 = blockIdx.x * kPartTok;
  const int c0 = blockIdx.y * kPartCols;
  const int H = a.hidden;
  __shared__ float red[8][kPartTok][M + 1];
  __shared__ float mix_s[kPartTok][kHcN + kHcN * kHcN];
  if (a.mode == 1) {
    for (int i = threadIdx.x; i < kPartTok * (kHcN + kHcN * kHcN); i += blockDim.x) {
      const int tt = i / (kHcN + kHcN * kHcN), j = i % (kHcN + kHcN * kHcN);
      mix_s[tt][j] = t0 + tt < a.rows ? a.mix_prev[(size_t)(t0 + tt) * (kHcN + kHcN * kHcN) + j] : 0.f;
    }
    __syncthreads();
  }
  float acc[kPartTok][M + 1];
#pragma unroll
  for (int tt = 0; tt < kPartTok; ++tt)
#pragma unroll
    for (int m = 0; m <= M; ++m) acc[tt][m] = 0.f;
  for (int c = c0 + threadIdx.x; c < c0 + kPartCols && c < H; c += blockDim.x) {
    float x[kPartTok][kHcN];
#pragma unroll
    for (int tt = 0; tt < kPartTok; ++tt) {
      const int t = t0 + tt;
#pragma unroll
      for (int i = 0; i < kHcN; ++i) x[tt][i] = 0.f;
      if (t >= a.rows) continue;
      float* xr = a.x + (size_t)t * kHcN * H;
      if (a.mode == 2) {
        const float e = __bfloat162float(a.embed[(size_t)a.ids[t] * H + c]);
#pragma unroll
        for (int i = 0; i < kHcN; ++i) {
          x[tt][i] = e;
          xr[(size_t)i * H + c] = e;
        }
      } else {
#pragma unroll
        for (int i = 0; i < kHcN; ++i) x[tt][i] = xr[(size_t)i * H + c];
        if (a.mode == 1) {
          const float y = bfr(a.y[(size_t)t * H + c]);
          float nx[kHcN];
#pragma unroll
          for (int i = 0; i < kHcN; ++i) {
            float v = mix_s[tt][i] * y;
#pragma unroll
            for (int j = 0; j < kHcN; ++j) v += mix_s[tt][kHcN + i * kHcN + j] * x[tt][j];
            nx[i] = v;
          }
#pragma unroll
          for (int i = 0; i < kHcN; ++i) {
            x[tt][i] = nx[i];
            xr[(size_t)i * H + c] = nx[i];
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kHcN; ++i) acc[tt][M] += x[tt][i] * x[tt][i];
    }
#pragma unroll
    for (int i = 0; i < kHcN; ++i)
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float w = __ldg(a.fn + (size_t)m * kHcN * H + (size_t)i * H + c);
#pragma unroll
        for (int tt = 0; tt < kPartTok; ++tt) acc[tt][m] += w * x[tt][i];
      }
  }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int tt = 0; tt < kPartTok; ++tt)
#pragma unroll
    for (int m = 0; m <= M; ++m) {
      const float v = warp_sum(acc[tt][m]);
      if (lane == 0) red[wid][tt][m] = v;
    }
  __syncthreads();
  for (int i = threadIdx.x; i < kPartTok * (M + 1); i += blockDim.x) {
    const int tt = i / (M + 1), m = i % (M + 1);
    if (t0 + tt >= a.rows) continue;
    float v = 0.f;
    for (int w = 0; w < 8; ++w) v += red[w][tt][m];
    a.partial[((size_t)(t0 + tt) * gridDim.y + blockIdx.y) * (M + 1) + m] = v;
  }
}

// Finalize one site for one row: mixing coefficients (pre, post, Sinkhorn residual), then
// h = pre @ X, RMSNorm (plain scale) and MXFP8 quantization of h.  head = 1: only the n
// pre logits exist (the final stream collapse).
template <int M>
__global__ void __launch_bounds__(256)
mhc_finalize_kernel(MhcFinalizeArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int t = blockIdx.x;
  const int H = a.hidden;
  __shared__ float mix[M + 1];
  __shared__ float pre_s[kHcN];
  __shared__ float red[32];
  if (threadIdx.x <= M) {
    float v = 0.f;
    for (int s = 0; s < a.slices; ++s) v += a.partial[((size_t)t * a.slices + s) * (M + 1) + threadIdx.x];
    mix[threadIdx.x] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float rs = rsqrtf(mix[M] / (float)(kHcN * H) + a.eps);
    for (int i = 0; i < kHcN; ++i) pre_s[i] = sigmoidf_(a.scale[0] * mix[i] * rs + a.base[i]);
    if (M == kHcM) {
      float* out = a.mix_out + (size_t)t * (kHcN + kHcN * kHcN);
      for (int i = 0; i < kHcN; ++i)
        out[i] = 2.f * sigmoidf_(a.scale[1] * mix[kHcN + i] * rs + a.base[kHcN + i]);
      float p[kHcN][kHcN];
      for (int i = 0; i < kHcN; ++i) {
        float mx = -INFINITY;
        for (int j = 0; j < kHcN; ++j) {
          p[i][j] = a.scale[2] * mix[2 * kHcN + i * kHcN + j] * rs + a.base[2 * kHcN + i * kHcN + j];
          mx = fmaxf(mx, p[i][j]);
        }
        float s = 0.f;
        for (int j = 0; j < kHcN; ++j) {
          p[i][j] = expf(p[i][j] - mx);
          s += p[i][j];
        }
        for (int j = 0; j < kHcN; ++j) p[i][j] /= s;
      }
      for (int it = 0; it < a.sinkhorn_iters; ++it) {
        for (int j = 0; j < kHcN; ++j) {
          float s = 0.f;
          for (int i = 0; i < kHcN; ++i) s += p[i][j];
          for (int i = 0; i < kHcN; ++i) p[i][j] /= s;
        }
        for (int i = 0; i < kHcN; ++i) {
          float s = 0.f;
          for (int j = 0; j < kHcN; ++j) s += p[i][j];
          for (int j = 0; j < kHcN; ++j) p[i][j] /= s;
        }
      }
      for (int i = 0; i < kHcN; ++i)
        for (int j = 0; j < kHcN; ++j) out[kHcN + i * kHcN + j] = p[i][j];
    }
  }
  __syncthreads();
  // h = pre @ X; each thread owns 8 consecutive columns per 2048-column pass.
  const float* xr = a.x + (size_t)t * kHcN * H;
  constexpr int kMaxPass = 4;  // H <= 8192
  float h[kMaxPass][8];
  float ss = 0.f;
  const int passes = (H + 2047) / 2048;
#pragma unroll
  for (int ps = 0; ps < kMaxPass; ++ps) {
    if (ps >= passes) break;
    const int col = ps * 2048 + threadIdx.x * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) h[ps][j] = 0.f;
    if (col < H) {
#pragma unroll
      for (int i = 0; i < kHcN; ++i) {
        const float4 u0 = *reinterpret_cast<const float4*>(xr + (size_t)i * H + col);
        const float4 u1 = *reinterpret_cast<const float4*>(xr + (size_t)i * H + col + 4);
        const float p = pre_s[i];
        h[ps][0] += p * u0.x; h[ps][1] += p * u0.y; h[ps][2] += p * u0.z; h[ps][3] += p * u0.w;
        h[ps][4] += p * u1.x; h[ps][5] += p * u1.y; h[ps][6] += p * u1.z; h[ps][7] += p * u1.w;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += h[ps][j] * h[ps][j];
    }
  }
  ss = block_sum_256(ss, red);
  const float rs = rsqrtf(ss / (float)H + a.eps);
#pragma unroll
  for (int ps = 0; ps < kMaxPass; ++ps) {
    if (ps >= passes) break;
    const int col = ps * 2048 + threadIdx.x * 8;
    const bool active = col < H;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = active ? h[ps][j] * rs * __bfloat162float(a.weight[col + j]) : 0.f;
    quant8_store(v, active, t, col, H, a.q, a.sf);
  }
}

// ------------------------------------------------------------------------------ norm + quant
// RMSNorm (plain scale) of a strided bf16 row slice, then MXFP8.  One CTA per row.
__global__ void __launch_bounds__(256)
rms_quant_kernel(const __nv_bfloat16* __restrict__ x, int ld_x, int width, const __nv_bfloat16* __restrict__ w,
                 float eps, uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  __shared__ float red[32];
  const int t = blockIdx.x;
  constexpr int kMaxPass = 4;
  float v[kMaxPass][8];
  float ss = 0.f;
  const int passes = (width + 2047) / 2048;
#pragma unroll
  for (int ps = 0; ps < kMaxPass; ++ps) {
    if (ps >= passes) break;
    const int col = ps * 2048 + threadIdx.x * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[ps][j] = 0.f;
    if (col < width) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)t * ld_x + col);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b[j]);
        v[ps][2 * j] = f.x;
        v[ps][2 * j + 1] = f.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[ps][j] * v[ps][j];
    }
  }
  ss = block_sum_256(ss, red);
  const float rs = rsqrtf(ss / (float)width + eps);
#pragma unroll
  for (int ps = 0; ps < kMaxPass; ++ps) {
    if (ps >= passes) break;
    const int col = ps * 2048 + threadIdx.x * 8;
    const bool active = col < width;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = active ? v[ps][j] * rs * __bfloat162float(w[col + j]) : 0.f;
    quant8_store(o, active, t, col, width, q, sf);
  }
}

// ------------------------------------------------------------------------------ MLA prologue
// One CTA per token: c_kv = rmsnorm(kv_a[:kl]) and k_pe = rope(kv_a[kl:]) into the latent
// cache, the index key rope(rmsnorm(wk x)) into the index cache, roped q_pe and index
// queries, and the scaled index-head weights.
__global__ void __launch_bounds__(256)
mla_prologue_kernel(MlaPrologueArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int pos = a.pos[t];
  const int slot = a.slot[t];
  const int page = a.page_table[(size_t)slot * a.max_pages + pos / a.page_size];
  const int off = pos % a.page_size;
  const __nv_bfloat16* pr = a.proj + (size_t)t * a.ld_proj;
  const int kl = a.kv_lora, R = a.rope, ID = a.index_dim;
  // c_kv (kl <= 512: 2 values per thread)
  {
    float v[2] = {0.f, 0.f};
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int c = threadIdx.x + j * 256;
      if (c < kl) {
        v[j] = __bfloat162float(pr[a.off_kva + c]);
        ss += v[j] * v[j];
      }
    }
    ss = block_sum_256(ss, red);
    const float rs = rsqrtf(ss / (float)kl + a.eps);
    __nv_bfloat16* row = a.ckv_cache + ((size_t)page * a.page_size + off) * (kl + R);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int c = threadIdx.x + j * 256;
      if (c < kl) row[c] = __float2bfloat16(v[j] * rs * __bfloat162float(a.kv_norm[c]));
    }
    if (threadIdx.x < R / 2) {
      const int i = threadIdx.x;
      float cs, sn;
      rope_cs(pos, i, R, a.theta, cs, sn);
      const float lo = __bfloat162float(pr[a.off_kva + kl + i]);
      const float hi = __bfloat162float(pr[a.off_kva + kl + i + R / 2]);
      row[kl + i] = __float2bfloat16(lo * cs - hi * sn);
      row[kl + i + R / 2] = __float2bfloat16(hi * cs + lo * sn);
    }
  }
  // index key: rmsnorm over ID (<= 256), bf16, then rope over the last R dims
  {
    __shared__ float kn[256];
    float v = threadIdx.x < ID ? __bfloat162float(pr[a.off_ik + threadIdx.x]) : 0.f;
    const float ss = block_sum_256(v * v, red);
    const float rs = rsqrtf(ss / (float)ID + a.eps);
    if (threadIdx.x < ID) kn[threadIdx.x] = bfr(v * rs * __bfloat162float(a.ik_norm[threadIdx.x]));
    __syncthreads();
    __nv_bfloat16* row = a.ik_cache + ((size_t)page * a.page_size + off) * ID;
    if (threadIdx.x < ID - R) row[threadIdx.x] = __float2bfloat16(kn[threadIdx.x]);
    if (threadIdx.x < R / 2) {
      const int i = threadIdx.x;
      float cs, sn;
      rope_cs(pos, i, R, a.theta, cs, sn);
      const float lo = kn[ID - R + i], hi = kn[ID - R + i + R / 2];
      row[ID - R + i] = __float2bfloat16(lo * cs - hi * sn);
      row[ID - R + i + R / 2] = __float2bfloat16(hi * cs + lo * sn);
    }
  }
  // q_pe of every local head; roped index queries
  const __nv_bfloat16* qr = a.qi + (size_t)t * a.ld_qi;
  const int half = R / 2;
  for (int i = threadIdx.x; i < (a.heads + a.index_heads) * half; i += blockDim.x) {
    const int h = i / half, d = i % half;
    float cs, sn;
    rope_cs(pos, d, R, a.theta, cs, sn);
    if (h < a.heads) {
      const __nv_bfloat16* src = qr + (size_t)h * a.qk_dim + a.nope;
      const float lo = __bfloat162float(src[d]), hi = __bfloat162float(src[d + half]);
      __nv_bfloat16* dst = a.q_pe + ((size_t)t * a.heads + h) * R;
      dst[d] = __float2bfloat16(lo * cs - hi * sn);
      dst[d + half] = __float2bfloat16(hi * cs + lo * sn);
    } else {
      const int ih = h - a.heads;
      const __nv_bfloat16* src = qr + a.off_iq + (size_t)ih * ID + (ID - R);
      const float lo = __bfloat162float(src[d]), hi = __bfloat162float(src[d + half]);
      __nv_bfloat16* dst = a.iq + ((size_t)t * a.index_heads + ih) * ID + (ID - R);
      dst[d] = __float2bfloat16(lo * cs - hi * sn);
      dst[d + half] = __float2bfloat16(hi * cs + lo * sn);
    }
  }
  for (int i = threadIdx.x; i < a.index_heads * (ID - R); i += blockDim.x) {
    const int ih = i / (ID - R), d = i % (ID - R);
    a.iq[((size_t)t * a.index_heads + ih) * ID + d] = qr[a.off_iq + (size_t)ih * ID + d];
  }
  for (int i = threadIdx.x; i < a.index_heads; i += blockDim.x)
    a.iw[(size_t)t * a.index_heads + i] = __bfloat162float(pr[a.off_iw + i]) * a.iw_scale;
}

// ------------------------------------------------------------------------------ absorb q
// q_lat[t, h, :] = W_UK[h]^T q_nope[t, h]: CTA per (head, 16 tokens), thread per 2
// latent columns.
constexpr int kAbsTok = 4;
__global__ void __launch_bounds__(256)
mla_absorb_q_kernel(const __nv_bfloat16* __restrict__ qi, int ld_qi, int qk_dim, int nope,
                    const __nv_bfloat16* __restrict__ w_uk, int kl, int heads, int rows,
                    __nv_bfloat16* __restrict__ q_lat) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int h = blockIdx.x;
  const int t0 = blockIdx.y * kAbsTok;
  __shared__ float qs[kAbsTok][128];
  for (int i = threadIdx.x; i < kAbsTok * nope; i += blockDim.x) {
    const int tt = i / nope, d = i % nope;
    qs[tt][d] = t0 + tt < rows ? __bfloat162float(qi[(size_t)(t0 + tt) * ld_qi + (size_t)h * qk_dim + d]) : 0.f;
  }
  __syncthreads();
  const int c = threadIdx.x * 2;
  if (c >= kl) return;
  float acc[kAbsTok][2];
#pragma unroll
  for (int tt = 0; tt < kAbsTok; ++tt) acc[tt][0] = acc[tt][1] = 0.f;
  const __nv_bfloat16* wh = w_uk + (size_t)h * nope * kl;
#pragma unroll 16
  for (int d = 0; d < nope; ++d) {
    const float2 w = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(wh + (size_t)d * kl + c));
#pragma unroll
    for (int tt = 0; tt < kAbsTok; ++tt) {
      acc[tt][0] += qs[tt][d] * w.x;
      acc[tt][1] += qs[tt][d] * w.y;
    }
  }
#pragma unroll
  for (int tt = 0; tt < kAbsTok; ++tt) {
    if (t0 + tt >= rows) break;
    *reinterpret_cast<__nv_bfloat162*>(q_lat + ((size_t)(t0 + tt) * heads + h) * kl + c) =
        __floats2bfloat162_rn(acc[tt][0], acc[tt][1]);
  }
}

// ------------------------------------------------------------------------------ MLA attention
// Split-KV decode/prefill over the selected keys of each token.  CTA per (token, split);
// keys are staged 32 at a time in shared memory; thread (key, head) pairs compute scores;
// an online softmax keeps per-head running max / sum; each thread accumulates 2 latent
// columns for every head.  Partial record per (token, head, split): o[kl] (unnormalised),
// m, l, 2 pad.
constexpr int kAttnKeys = 32;
constexpr int kMaxHeads = 16;
constexpr int kLat = 512;
constexpr int kRope = 64;
constexpr int kRowPad = kLat + kRope + 8;  // bf16 elements per staged key row (bank spread)
constexpr int kQPad = kLat + kRope + 4;    // floats per staged query row

__global__ void __launch_bounds__(256)
mla_attn_kernel(MlaAttnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* qs = reinterpret_cast<float*>(smem_raw);                                   // [heads][kQPad]
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(qs + a.heads * kQPad);        // [kAttnKeys][kRowPad]
  float* ps = reinterpret_cast<float*>(ks + kAttnKeys * kRowPad);                    // [heads][kAttnKeys]
  __shared__ float m_s[kMaxHeads], l_s[kMaxHeads], scale_s[kMaxHeads];
  const int t = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  const int HL = a.heads;
  const int n_keys = a.n_sel[t];
  const int per = (n_keys + S - 1) / S;
  const int k0 = split * per, k1 = min(n_keys, k0 + per);
  const int slot = a.slot[t];
  for (int i = threadIdx.x; i < HL * (kLat + kRope); i += blockDim.x) {
    const int h = i / (kLat + kRope), d = i % (kLat + kRope);
    qs[h * kQPad + d] = d < kLat ? __bfloat162float(a.q_lat[((size_t)t * HL + h) * kLat + d])
                                 : __bfloat162float(a.q_pe[((size_t)t * HL + h) * kRope + d - kLat]);
  }
  if (threadIdx.x < kMaxHeads) {
    m_s[threadIdx.x] = -INFINITY;
    l_s[threadIdx.x] = 0.f;
  }
  float acc[kMaxHeads][2];
#pragma unroll
  for (int h = 0; h < kMaxHeads; ++h) acc[h][0] = acc[h][1] = 0.f;
  const int* sel = a.sel + (size_t)t * a.ld_sel;
  for (int kb = k0; kb < k1; kb += kAttnKeys) {
    const int nk = min(kAttnKeys, k1 - kb);
    __syncthreads();
    // stage nk key rows (72 x 16 B each)
    for (int i = threadIdx.x; i < nk * 72; i += blockDim.x) {
      const int kk = i / 72, piece = i % 72;
      const int p = sel[kb + kk];
      const int page = a.page_table[(size_t)slot * a.max_pages + p / a.page_size];
      const uint4* src = reinterpret_cast<const uint4*>(a.ckv_cache + ((size_t)page * a.page_size + p % a.page_size) *
                                                                          (kLat + kRope));
      *reinterpret_cast<uint4*>(ks + kk * kRowPad + piece * 8) = src[piece];
    }
    __syncthreads();
    // scores: pairs (key, head)
    for (int i = threadIdx.x; i < nk * HL; i += blockDim.x) {
      const int kk = i % nk, h = i / nk;
      const __nv_bfloat16* kr = ks + kk * kRowPad;
      const float* qr = qs + h * kQPad;
      float s = 0.f;
#pragma unroll 4
      for (int d = 0; d < kLat + kRope; d += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(kr + d);
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
        const float4 q0 = *reinterpret_cast<const float4*>(qr + d);
        const float4 q1 = *reinterpret_cast<const float4*>(qr + d + 4);
        float2 f;
        f = __bfloat1622float2(b[0]); s += q0.x * f.x + q0.y * f.y;
        f = __bfloat1622float2(b[1]); s += q0.z * f.x + q0.w * f.y;
        f = __bfloat1622float2(b[2]); s += q1.x * f.x + q1.y * f.y;
        f = __bfloat1622float2(b[3]); s += q1.z * f.x + q1.w * f.y;
      }
      ps[h * kAttnKeys + kk] = s * a.sm_scale;
    }
    __syncthreads();
    // per-head online softmax update (warp per head)
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int h = wid; h < HL; h += blockDim.x / 32) {
      const float s = lane < nk ? ps[h * kAttnKeys + lane] : -INFINITY;
      const float mx = warp_max(s);
      const float m_new = fmaxf(m_s[h], mx);
      const float p = lane < nk ? expf(s - m_new) : 0.f;
      const float sum = warp_sum(p);
      if (lane < kAttnKeys) ps[h * kAttnKeys + lane] = p;
      __syncwarp();
      if (lane == 0) {
        const float sc = expf(m_s[h] - m_new);
        scale_s[h] = sc;
        l_s[h] = l_s[h] * sc + sum;
        m_s[h] = m_new;
      }
    }
    __syncthreads();
    const int c = threadIdx.x * 2;
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h >= HL) break;
      const float sc = scale_s[h];
      acc[h][0] *= sc;
      acc[h][1] *= sc;
    }
    for (int kk = 0; kk < nk; ++kk) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(ks + kk * kRowPad + c));
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) {
        if (h >= HL) break;
        const float p = ps[h * kAttnKeys + kk];
        acc[h][0] += p * v.x;
        acc[h][1] += p * v.y;
      }
    }
  }
  __syncthreads();
  const int c = threadIdx.x * 2;
#pragma unroll
  for (int h = 0; h < kMaxHeads; ++h) {
    if (h >= HL) break;
    float* rec = a.partial + (((size_t)t * HL + h) * S + split) * (kLat + 4);
    rec[c] = acc[h][0];
    rec[c + 1] = acc[h][1];
    if (threadIdx.x == 0) {
      rec[kLat] = m_s[h];
      rec[kLat + 1] = l_s[h];
    }
  }
}

// ------------------------------------------------------------------------------ value up-proj
// Merge the split records of (token, head) into o_lat (bf16-rounded), then
// o[t, h, :] = W_UV[h] o_lat (bf16) and MXFP8-quantize the row [heads * v] for o_proj.
// CTA per (head, 8 tokens); 128 threads, thread per value dim.
constexpr int kUpTok = 2;
__global__ void __launch_bounds__(128)
mla_up_kernel(MlaUpArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int h = blockIdx.x;
  const int t0 = blockIdx.y * kUpTok;
  const int HL = a.heads, S = a.splits, V = a.v_dim;
  __shared__ float ol[kUpTok][kLat];
  __shared__ float wgt[kUpTok][64];
  // merge weights per (token, split)
  for (int i = threadIdx.x; i < kUpTok; i += blockDim.x) {
    const int t = t0 + i;
    if (t >= a.rows) continue;
    const float* base = a.partial + (((size_t)t * HL + h) * S) * (kLat + 4);
    float m = -INFINITY;
    for (int s = 0; s < S; ++s) m = fmaxf(m, base[(size_t)s * (kLat + 4) + kLat]);
    float l = 0.f;
    for (int s = 0; s < S; ++s) {
      const float ms = base[(size_t)s * (kLat + 4) + kLat];
      const float w = ms == -INFINITY ? 0.f : expf(ms - m);
      wgt[i][s] = w;
      l += w * base[(size_t)s * (kLat + 4) + kLat + 1];
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    for (int s = 0; s < S; ++s) wgt[i][s] *= inv;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kUpTok * kLat; i += blockDim.x) {
    const int tt = i / kLat, c = i % kLat;
    const int t = t0 + tt;
    float v = 0.f;
    if (t < a.rows) {
      const float* base = a.partial + (((size_t)t * HL + h) * S) * (kLat + 4);
      for (int s = 0; s < S; ++s) v += wgt[tt][s] * base[(size_t)s * (kLat + 4) + c];
    }
    ol[tt][c] = bfr(v);
  }
  __syncthreads();
  const int d = threadIdx.x;  // value dim (V == 128)
  float acc[kUpTok];
#pragma unroll
  for (int tt = 0; tt < kUpTok; ++tt) acc[tt] = 0.f;
  const __nv_bfloat16* wh = a.w_uv_t + (size_t)h * kLat * V;
#pragma unroll 16
  for (int c = 0; c < kLat; ++c) {
    const float w = __bfloat162float(wh[(size_t)c * V + d]);
#pragma unroll
    for (int tt = 0; tt < kUpTok; ++tt) acc[tt] += ol[tt][c] * w;
  }
  const int width = HL * V;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int tt = 0; tt < kUpTok; ++tt) {
    const int t = t0 + tt;
    if (t >= a.rows) break;  // uniform across the CTA
    const float o = bfr(acc[tt]);
    const float amax = warp_max(fabsf(o));
    const uint8_t code = mx_scale_e8m0(amax);
    const int col = h * V + d;
    a.q[(size_t)t * width + col] = f32_to_e4m3(o * mx_inv_scale(code));
    if (lane == 0) {
      const int kb = col >> 5;
      a.sf[((size_t)(t >> 7) * (width >> 7) + (kb >> 2)) * 512 + sf_atom_offset(t & 127, kb & 3)] = code;
    }
  }
}

// ------------------------------------------------------------------------------ DSA indexer
constexpr int kIdxDim = 128;

// Tensor-core indexer scores: per (token, 1024-key chunk) CTA, 128-key tiles are staged
// by cp.async into the K-major 128-byte-swizzled layout (two 64-dim chunks per row), one
// thread issues 8 tcgen05.mma (kind::f16, bf16, M = 128 keys, N = index heads, K = 16
// each) into TMEM, and each of the 4 warps reads its 32 keys' head scores back to form
// sum_h w_h relu(q_h . k) * scale.  The next tile's copies overlap the MMA and epilogue.
constexpr int kTcKeys = 128;
constexpr int kTcTiles = 8;

ZS_DEVICE void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
ZS_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
ZS_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Byte offset of 16-byte piece p (0..15) of row r in a K-major SW128 tile of `rows` rows
// whose 256-byte rows are split into two 64-element chunks.
ZS_DEVICE uint32_t sw128_off(int r, int p, int rows) {
  return (uint32_t)((p >> 3) * rows * 128 + r * 128 + (((p & 7) ^ (r & 7)) << 4));
}

template <int IH>
__global__ void __launch_bounds__(128)
dsa_scores_tc_kernel(DsaScoresArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int t = blockIdx.x;
  const int ctx = a.ctx_len[t];
  const int s_begin = blockIdx.y * kTcKeys * kTcTiles;
  if (ctx <= a.topk || s_begin >= ctx) return;  // uniform: before any barrier or TMEM use
  const int n_tiles = min(kTcTiles, (ctx - s_begin + kTcKeys - 1) / kTcKeys);
  extern __shared__ __align__(1024) uint8_t tc_scores_smem[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_scores_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* A = base;                                  // [2][2 chunks][128 rows][128 B]
  uint8_t* B = base + 2 * 2 * kTcKeys * 128;          // [2 chunks][IH rows][128 B]
  float* wsm = reinterpret_cast<float*>(B + 2 * IH * 128);
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr uint32_t kCols = IH < 32 ? 32 : IH;
  if (warp == 0) {
    tmem_alloc(&tmem_base, kCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&mbar, 1);
    fence_barrier_init();
  }
  // Index queries (B operand) and head weights.
  const __nv_bfloat16* q = a.iq + (size_t)t * IH * kIdxDim;
  for (int i = tid; i < IH * 16; i += blockDim.x) {
    const int h = i >> 4, p = i & 15;
    cp_async16(B + sw128_off(h, p, IH), q + (size_t)h * kIdxDim + p * 8);
  }
  for (int i = tid; i < IH; i += blockDim.x) wsm[i] = a.iw[(size_t)t * IH + i];
  const int slot = a.slot[t];
  auto stage_tile = [&](int tile, uint8_t* dst) {
    const int s0 = s_begin + tile * kTcKeys;
    for (int i = tid; i < kTcKeys * 16; i += blockDim.x) {
      const int r = i >> 4, p = i & 15;
      const int s = s0 + r;
      uint8_t* d = dst + sw128_off(r, p, kTcKeys);
      if (s < ctx) {
        const int page = a.page_table[(size_t)slot * a.max_pages + s / a.page_size];
        cp_async16(d, a.ik_cache + ((size_t)page * a.page_size + s % a.page_size) * kIdxDim + p * 8);
      } else {
        *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
      }
    }
  };
  stage_tile(0, A);
  cp_async_commit();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t idesc = make_idesc_bf16(kTcKeys, IH, 0, 0);
  bool ok = true;
  for (int i = 0; i < n_tiles; ++i) {
    cp_async_wait_all();
    fence_proxy_async_shared();
    __syncthreads();
    uint8_t* Ai = A + (i & 1) * (2 * kTcKeys * 128);
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kc = 0; kc < 2; ++kc)
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          const uint64_t ad = make_smem_desc(smem_u32(Ai + kc * kTcKeys * 128) + kb * 32, 16, 1024, 2);
          const uint64_t bd = make_smem_desc(smem_u32(B + kc * IH * 128) + kb * 32, 16, 1024, 2);
          mma_bf16(tmem, ad, bd, idesc, (kc | kb) != 0 ? 1u : 0u);
        }
      tc_commit(&mbar);
    }
    if (i + 1 < n_tiles) {
      stage_tile(i + 1, A + ((i + 1) & 1) * (2 * kTcKeys * 128));
      cp_async_commit();
    }
    ok = mbar_wait(&mbar, (uint32_t)(i & 1), a.err);
    if (!__syncthreads_and(ok)) break;  // bounded wait gave up: the error is recorded
    tc_fence_after();
    const uint32_t tq = tmem + ((uint32_t)(warp * 32) << 16);
    float score = 0.f;
#pragma unroll
    for (int c0 = 0; c0 < IH; c0 += (IH < 32 ? 16 : 32)) {
      if (IH < 32) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tq + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) score += wsm[c0 + j] * fmaxf(__uint_as_float(r[j]), 0.f);
      } else {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tq + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) score += wsm[c0 + j] * fmaxf(__uint_as_float(r[j]), 0.f);
      }
    }
    const int s = s_begin + i * kTcKeys + warp * 32 + lane;
    if (s < ctx) a.scores[(size_t)t * a.ld_scores + s] = score * a.scale;
    tc_fence_before();
    __syncthreads();
  }
  cp_async_wait_all();  // no copy may still target shared memory when the CTA exits
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

// Top-k selection per token (CTA of 1024 threads): positions 0..ctx-1 when ctx <= k, else
// the k highest scores, ties to the lower position, emitted in ascending position order.
// Radix select over the order-preserving 32-bit image of the scores (4 passes of 8 bits),
// then a two-scan compaction (strictly greater, then the leading ties).
ZS_DEVICE uint32_t ord_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(1024)
dsa_topk_kernel(DsaTopkArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int t = blockIdx.x;
  const int ctx = a.ctx_len[t];
  const int K = a.topk;
  int* out = a.sel + (size_t)t * a.ld_sel;
  if (ctx <= K) {
    for (int i = threadIdx.x; i < ctx; i += blockDim.x) out[i] = i;
    if (threadIdx.x == 0) a.n_sel[t] = ctx;
    return;
  }
  const float* sc = a.scores + (size_t)t * a.ld_scores;
  __shared__ int hist[256];
  __shared__ uint32_t prefix_s;
  __shared__ int need_s;
  if (threadIdx.x == 0) {
    prefix_s = 0;
    need_s = K;  // rank (1-based) of the threshold among keys matching the prefix
  }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = prefix_s;
    const uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
    for (int i = threadIdx.x; i < ctx; i += blockDim.x) {
      const uint32_t k = ord_key(sc[i]);
      if ((k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFF], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int need = need_s;
      int d = 255;
      for (; d > 0; --d) {
        if (hist[d] >= need) break;
        need -= hist[d];
      }
      prefix_s = prefix | ((uint32_t)d << shift);
      need_s = need;
    }
    __syncthreads();
  }
  const uint32_t thr = prefix_s;
  const int ties_taken = need_s;  // how many keys equal to thr are selected (lowest positions)
  // Compaction in position order: each thread owns a contiguous chunk.
  __shared__ int cnt_gt[1024], cnt_eq[1024];
  const int chunk = (ctx + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * chunk, b1 = min(ctx, b0 + chunk);
  int ng = 0, ne = 0;
  for (int i = b0; i < b1; ++i) {
    const uint32_t k = ord_key(sc[i]);
    ng += k > thr;
    ne += k == thr;
  }
  cnt_gt[threadIdx.x] = ng;
  cnt_eq[threadIdx.x] = ne;
  __syncthreads();
  if (threadIdx.x == 0) {  // exclusive scans (1024 entries; one thread is enough here)
    int sg = 0, se = 0;
    for (int i = 0; i < (int)blockDim.x; ++i) {
      const int g = cnt_gt[i], e = cnt_eq[i];
      cnt_gt[i] = sg;
      cnt_eq[i] = se;
      sg += g;
      se += e;
    }
  }
  __syncthreads();
  // Output index of a selected key = (# selected keys before it) = greater-before +
  // min(ties-before, ties_taken).
  int g_before = cnt_gt[threadIdx.x], e_before = cnt_eq[threadIdx.x];
  for (int i = b0; i < b1; ++i) {
    const uint32_t k = ord_key(sc[i]);
    if (k > thr) {
      out[g_before + min(e_before, ties_taken)] = i;
      ++g_before;
    } else if (k == thr) {
      if (e_before < ties_taken) out[g_before + e_before] = i;
      ++e_before;
    }
  }
  if (threadIdx.x == 0) a.n_sel[t] = K;
}

// ------------------------------------------------------------------------------ MoE combine
// y[t, :] = sum_j w[t, j] * expert_rows[src[t, j], :] (fp32, fixed term order).
__global__ void __launch_bounds__(256)
gather_sum_kernel(const __nv_bfloat16* __restrict__ rows_in, const int* __restrict__ src,
                  const float* __restrict__ w, int k1, int hidden, float* __restrict__ y) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < hidden; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k1; ++j) {
      const int r = src[(size_t)t * k1 + j];
      if (r < 0) continue;
      const float wt = w[(size_t)t * k1 + j];
      const uint4 u = *reinterpret_cast<const uint4*>(rows_in + (size_t)r * hidden + c);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(b[q]);
        acc[2 * q] += f.x * wt;
        acc[2 * q + 1] += f.y * wt;
      }
    }
    float4* dst = reinterpret_cast<float4*>(y + (size_t)t * hidden + c);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// ------------------------------------------------------------------------------ MLA on tensor cores
// Tensor-core form of mla_attn_kernel (same partial records).  CTA of 4 warps per (token,
// split); the split's selected keys go through 128-key tiles:
//   * Gather: every key row (576 bf16: 512 latent + 64 rope) is copied by cp.async, 16 bytes
//     at a time, into a K-major 128-byte-swizzled tile image [9 dim chunks][128 keys][128 B]
//     (rows of a tile come from arbitrary pages, so no bulk copy can place them); rows past
//     the split's keys are zeroed.
//   * S^T = K Q^T: one thread issues 36 tcgen05.mma (kind::f16, bf16, M = 128 keys, N = 16
//     head slots, K = 16 dims each) into TMEM columns 0-15.  Q = [q_lat | q_pe] per head.
//   * Online softmax in the exp2 domain exactly as the paged decode kernel: thread t owns
//     key t, per-head maxima / sums through shared memory, P stored bf16 K-major, the
//     running O rescaled in TMEM.
//   * O^T += C^T P^T with the same tile image read MN-major (the latent part of a key row
//     is its value row): 4 x 8 MMAs (M = 128 latent dims, N = 16, K = 16 keys) into TMEM
//     columns 16-79.
// The image is single-buffered (147 KiB): the next tile's gather starts once this tile's
// second product has consumed it.
constexpr int kMtKeys = 128;
constexpr int kMtChunks = (kLat + kRope) / 64;       // 9
constexpr int kMtPlane = kMtKeys * 128;              // bytes per 64-dim chunk plane
constexpr int kMtN = 16;                             // head slots (heads <= 16)

struct MlaTcSmem {
  uint8_t k[kMtChunks * kMtPlane];   // key tile image (1024-aligned: first member)
  uint8_t q[kMtChunks][kMtN * 128];  // [q_lat | q_pe] per head slot, slots >= heads zero
  uint8_t p[2][kMtN * 128];          // P: [16 slots][128 keys] K-major, 2 chunks of 64 keys
  float red_max[4][kMtN];
  float red_sum[4][kMtN];
  float m[kMtN], l[kMtN], r[kMtN];
  uint64_t mma1, mma2;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(128, 1)
mla_attn_tc_kernel(MlaAttnArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t mla_tc_smem_raw[];
  MlaTcSmem& s = *reinterpret_cast<MlaTcSmem*>((reinterpret_cast<uintptr_t>(mla_tc_smem_raw) + 1023) & ~uintptr_t(1023));
  const int t = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int HL = a.heads;
  const int n_keys = a.n_sel[t];
  const int per = (n_keys + S - 1) / S;
  const int k0 = min(n_keys, split * per), k1 = min(n_keys, k0 + per);
  const int nk_all = k1 - k0;
  const int ntiles = (nk_all + kMtKeys - 1) / kMtKeys;
  const float qscale = a.sm_scale * 1.4426950408889634f;  // exp2 domain
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, 128);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&s.mma1, 1);
    mbar_init(&s.mma2, 1);
    fence_barrier_init();
  }
  if (tid < kMtN) {
    s.m[tid] = -INFINITY;
    s.l[tid] = 0.f;
  }
  for (int i = tid; i < kMtN * (kLat + kRope) / 8; i += blockDim.x) {
    const int h = i / 72, piece = i % 72, c = piece >> 3, j = piece & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < HL)
      v = piece < 64 ? *reinterpret_cast<const uint4*>(a.q_lat + ((size_t)t * HL + h) * kLat + piece * 8)
                     : *reinterpret_cast<const uint4*>(a.q_pe + ((size_t)t * HL + h) * kRope + (piece - 64) * 8);
    *reinterpret_cast<uint4*>(s.q[c] + h * 128 + ((j ^ (h & 7)) << 4)) = v;
  }
  fence_proxy_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t t_s = tmem, t_o = tmem + kMtN;
  const int* sel = a.sel + (size_t)t * a.ld_sel + k0;
  const int* pt = a.page_table + (size_t)a.slot[t] * a.max_pages;
  bool ok = true;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int kb = tile * kMtKeys;
    const int nk = min(kMtKeys, nk_all - kb);
    // Gather: warp w copies keys w, w + 4, ...; a row's 72 pieces spread over the lanes.
    for (int kk = warp; kk < kMtKeys; kk += 4) {
      uint8_t* rowbase = s.k + kk * 128;
      if (kk < nk) {
        const int pos = __ldg(sel + kb + kk);
        const int page = __ldg(pt + pos / a.page_size);
        const uint8_t* src = reinterpret_cast<const uint8_t*>(
            a.ckv_cache + ((size_t)page * a.page_size + pos % a.page_size) * (kLat + kRope));
        for (int piece = lane; piece < 72; piece += 32)
          cp_async16(rowbase + (piece >> 3) * kMtPlane + (((piece & 7) ^ (kk & 7)) << 4), src + piece * 16);
      } else {
        for (int piece = lane; piece < 72; piece += 32)
          *reinterpret_cast<uint4*>(rowbase + (piece >> 3) * kMtPlane + (((piece & 7) ^ (kk & 7)) << 4)) =
              make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
    cp_async_wait_all();
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = make_idesc_bf16(kMtKeys, kMtN, 0, 0);
#pragma unroll
      for (int c = 0; c < kMtChunks; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ad = make_smem_desc(smem_u32(s.k + c * kMtPlane) + k * 32, 16, 1024, 2);
          const uint64_t bd = make_smem_desc(smem_u32(s.q[c]) + k * 32, 16, 1024, 2);
          mma_bf16(t_s, ad, bd, idesc, (c | k) ? 1u : 0u);
        }
      tc_commit(&s.mma1);
    }
    ok = mbar_wait(&s.mma1, (uint32_t)(tile & 1), a.err);
    if (!__syncthreads_and(ok)) break;
    tc_fence_after();
    // ---- online softmax: thread tid owns key tid of the tile
    uint32_t sr[16];
    tmem_ld_32x32b_x16(t_s + lane_off, sr);
    tmem_ld_wait();
    const bool valid = tid < nk;
    float sv[kMtN];
#pragma unroll
    for (int h = 0; h < kMtN; ++h) sv[h] = (valid && h < HL) ? __uint_as_float(sr[h]) * qscale : -INFINITY;
#pragma unroll
    for (int h = 0; h < kMtN; ++h) {
      const float v = warp_max(sv[h]);
      if (lane == 0) s.red_max[warp][h] = v;
    }
    __syncthreads();
    float mnew[kMtN];
#pragma unroll
    for (int h = 0; h < kMtN; ++h)
      mnew[h] = fmaxf(fmaxf(s.m[h], fmaxf(s.red_max[0][h], s.red_max[1][h])), fmaxf(s.red_max[2][h], s.red_max[3][h]));
    {
      const int chunk = tid >> 6, within = tid & 63, piece = within >> 3, sub = (within & 7) * 2;
#pragma unroll
      for (int h = 0; h < kMtN; ++h) {
        const float pv = sv[h] == -INFINITY ? 0.f : exp2f(sv[h] - mnew[h]);
        const __nv_bfloat16 pb = __float2bfloat16_rn(pv);
        *reinterpret_cast<__nv_bfloat16*>(s.p[chunk] + h * 128 + ((piece ^ (h & 7)) << 4) + sub) = pb;
        const float sum = warp_sum(__bfloat162float(pb));
        if (lane == 0) s.red_sum[warp][h] = sum;
      }
    }
    fence_proxy_async_shared();
    __syncthreads();
    if (tid < kMtN) {
      const int h = tid;
      const float mo = s.m[h];
      const float rr = mo == -INFINITY ? 0.f : exp2f(mo - mnew[h]);
      s.l[h] = s.l[h] * rr + (s.red_sum[0][h] + s.red_sum[1][h] + s.red_sum[2][h] + s.red_sum[3][h]);
      s.m[h] = mnew[h];
      s.r[h] = rr;
    }
    __syncthreads();
    if (tile > 0) {  // rescale the running O^T (TMEM lane = latent dim, column = head slot)
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t o[16];
        tmem_ld_32x32b_x16(t_o + mt * kMtN + lane_off, o);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 16; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * s.r[h]);
        tmem_st_32x32b_x16(t_o + mt * kMtN + lane_off, o);
      }
      tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc2 = make_idesc_bf16(128, kMtN, 1, 0);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          // A: latent dims 128 mt.. (chunks 2mt, 2mt+1, LBO = one chunk plane) x keys
          // 16 ks.. (two 8-key groups, SBO = 1 KiB), MN-major.
          const uint64_t ad = make_smem_desc(smem_u32(s.k + 2 * mt * kMtPlane) + ks * 16 * 128, kMtPlane, 1024, 2);
          const uint64_t bd = make_smem_desc(smem_u32(s.p[ks >> 2]) + (ks & 3) * 32, 16, 1024, 2);
          mma_bf16(t_o + mt * kMtN, ad, bd, idesc2, (tile > 0 || ks > 0) ? 1u : 0u);
        }
      tc_commit(&s.mma2);
    }
    ok = mbar_wait(&s.mma2, (uint32_t)(tile & 1), a.err);
    if (!__syncthreads_and(ok)) break;
    tc_fence_after();
  }
  const int h_lim = HL < kMtN ? HL : kMtN;
  if (ok) {
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      uint32_t o[16];
      if (ntiles > 0) {
        tmem_ld_32x32b_x16(t_o + mt * kMtN + lane_off, o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) o[h] = 0u;
      }
      const int dim = mt * 128 + tid;
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        if (h >= h_lim) break;
        a.partial[(((size_t)t * HL + h) * S + split) * (kLat + 4) + dim] = __uint_as_float(o[h]);
      }
    }
    if (tid < h_lim) {
      float* rec = a.partial + (((size_t)t * HL + tid) * S + split) * (kLat + 4);
      // Records hold the natural-log maximum (the SIMT kernel's convention).
      rec[kLat] = s.m[tid] == -INFINITY ? -INFINITY : s.m[tid] * 0.6931471805599453f;
      rec[kLat + 1] = s.l[tid];
    }
  } else if (tid < h_lim) {
    // Abort (the error word is set): an empty record, so the merge skips this split.
    float* rec = a.partial + (((size_t)t * HL + tid) * S + split) * (kLat + 4);
    rec[kLat] = -INFINITY;
    rec[kLat + 1] = 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace ds
}  // namespace zs

// ------------------------------------------------------------------------------ host API
namespace ds = zs::ds;

int zs_mhc_partial(const MhcPartialArgs* a, cudaStream_t stream) {
  if (a->rows <= 0) return 0;
  if (a->hidden % 8 != 0 || (a->m != ds::kHcM && a->m != ds::kHcN)) return -2;
  dim3 grid((a->rows + ds::kPartTok - 1) / ds::kPartTok, (a->hidden + ds::kPartCols - 1) / ds::kPartCols);
  if (a->m == ds::kHcM) zs_launch(ds::mhc_partial_kernel<ds::kHcM>, grid, 256, 0, stream, *a);
  else zs_launch(ds::mhc_partial_kernel<ds::kHcN>, grid, 256, 0, stream, *a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_mhc_slices(int hidden) { return (hidden + ds::kPartCols - 1) / ds::kPartCols; }

int zs_mhc_finalize(const MhcFinalizeArgs* a, cudaStream_t stream) {
  if (a->rows <= 0) return 0;
  if (a->hidden % 32 != 0 || a->hidden > 8192) return -2;
  if (a->m == ds::kHcM) zs_launch(ds::mhc_finalize_kernel<ds::kHcM>, a->rows, 256, 0, stream, *a);
  else if (a->m == ds::kHcN) zs_launch(ds::mhc_finalize_kernel<ds::kHcN>, a->rows, 256, 0, stream, *a);
  else return -2;
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_rms_quant(const void* x, int ld_x, int width, const void* w, float eps, int rows, uint8_t* q, uint8_t* sf,
                 cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (width % 32 != 0 || width > 8192 || ld_x % 8 != 0) return -2;
  zs_launch(ds::rms_quant_kernel, rows, 256, 0, stream, static_cast<const __nv_bfloat16*>(x), ld_x, width,
                                                 static_cast<const __nv_bfloat16*>(w), eps, q, sf);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_mla_prologue(const MlaPrologueArgs* a, cudaStream_t stream) {
  if (a->rows <= 0) return 0;
  if (a->kv_lora > 512 || a->index_dim > 256 || a->rope > 2 * 256 || a->rope % 2 != 0) return -2;
  zs_launch(ds::mla_prologue_kernel, a->rows, 256, 0, stream, *a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_mla_absorb_q(const void* qi, int ld_qi, int qk_dim, int nope, const void* w_uk, int kl, int heads, int rows,
                    void* q_lat, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (nope > 128 || kl > 512 || kl % 2 != 0) return -2;
  dim3 grid(heads, (rows + ds::kAbsTok - 1) / ds::kAbsTok);
  zs_launch(ds::mla_absorb_q_kernel, grid, 256, 0, stream,
      static_cast<const __nv_bfloat16*>(qi), ld_qi, qk_dim, nope, static_cast<const __nv_bfloat16*>(w_uk), kl, heads,
      rows, static_cast<__nv_bfloat16*>(q_lat));
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

size_t zs_mla_attn_smem(int heads) {
  return (size_t)heads * ds::kQPad * 4 + (size_t)ds::kAttnKeys * ds::kRowPad * 2 + (size_t)heads * ds::kAttnKeys * 4;
}

int zs_mla_attn(const MlaAttnArgs* a, cudaStream_t stream) {
  if (a->rows <= 0) return 0;
  if (a->heads > ds::kMaxHeads || a->kv_lora != ds::kLat || a->rope != ds::kRope || a->splits < 1 ||
      a->splits > 64)
    return -2;
  if (a->impl == 2) {  // tensor cores (heads <= 16 as checked above)
    const size_t smem = sizeof(ds::MlaTcSmem) + 1024;
    static bool tc_attr_set = false;
    if (!tc_attr_set) {
      cudaFuncSetAttribute(ds::mla_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      tc_attr_set = true;
    }
    zs_launch(ds::mla_attn_tc_kernel, dim3(a->rows, a->splits), 128, smem, stream, *a);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
  }
  const size_t smem = zs_mla_attn_smem(a->heads);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(ds::mla_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    attr_set = true;
  }
  dim3 grid(a->rows, a->splits);
  zs_launch(ds::mla_attn_kernel, grid, 256, smem, stream, *a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_mla_up(const MlaUpArgs* a, cudaStream_t stream) {
  if (a->rows <= 0) return 0;
  if (a->v_dim != 128 || a->splits > 64 || (a->heads * a->v_dim) % 128 != 0) return -2;
  dim3 grid(a->heads, (a->rows + ds::kUpTok - 1) / ds::kUpTok);
  zs_launch(ds::mla_up_kernel, grid, 128, 0, stream, *a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_dsa_scores(const DsaScoresArgs* a, int max_ctx, cudaStream_t stream) {
  if (a->rows <= 0 || max_ctx <= a->topk) return 0;
  const int ih = a->index_heads;
  if (ih != 16 && ih != 32 && ih != 64 && ih != 128) return -2;
  const size_t smem = 1024 + 2 * 2 * ds::kTcKeys * 128 + 2 * (size_t)ih * 128 + (size_t)ih * 4;
  dim3 grid(a->rows, (max_ctx + ds::kTcKeys * ds::kTcTiles - 1) / (ds::kTcKeys * ds::kTcTiles));
  auto launch = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    zs_launch(kern, grid, 128, smem, stream, *a);
  };
  if (ih == 16) launch(ds::dsa_scores_tc_kernel<16>);
  else if (ih == 32) launch(ds::dsa_scores_tc_kernel<32>);
  else if (ih == 64) launch(ds::dsa_scores_tc_kernel<64>);
  else launch(ds::dsa_scores_tc_kernel<128>);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_dsa_topk(const DsaTopkArgs* a, cudaStream_t stream) {
  if (a->rows <= 0) return 0;
  zs_launch(ds::dsa_topk_kernel, a->rows, 1024, 0, stream, *a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int zs_gather_sum(const void* rows_in, const int* src, const float* w, int k1, int hidden, int rows, float* y,
                  cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (hidden % 8 != 0) return -2;
  zs_launch(ds::gather_sum_kernel, rows, 256, 0, stream, static_cast<const __nv_bfloat16*>(rows_in), src, w, k1, hidden, y);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

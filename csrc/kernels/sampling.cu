// Full-distribution sampling on the GPU: penalties, temperature, top-k, top-p, a seeded
// draw, and log-probabilities, over fp32 logits of the whole vocabulary (one CTA of 1024
// threads per row).  The fused lm_head epilogue covers greedy and plain temperature
// sampling without materialising logits; this kernel serves the rows that need more.
//
//  * penalties (OpenAI presence / frequency, multiplicative repetition): the row's token
//    history is sorted in shared memory, each distinct token adjusts its logit once
//    (repetition: positive logits divided, negative multiplied; then - frequency * count
//    - presence), in place in the logits buffer;
//  * greedy rows (temperature <= 0): argmax of the penalised logits, smallest id on ties;
//  * stochastic rows: s = logit / T.  Top-k keeps the k largest s (radix select over the
//    order-preserving image of s, 4-bit digits; every token tied with the k-th value is
//    kept).  Top-p keeps tokens in descending order while the probability mass before
//    them is below p (mass-weighted radix select; ties at the boundary value kept).  The
//    draw u = SplitMix64(seed) in [0, 1) picks the token where the kept mass, summed in
//    token-id order, first exceeds u * (kept mass): a sample of the same truncated
//    distribution as an inverse CDF in sorted order.  Every mass is a fixed-order
//    reduction (per-thread contiguous chunks, then a tree), so a seed reproduces its
//    token bit for bit.
//  * log-probabilities of the raw logits: the chosen token's and the top-N (N <= 5).
//
// Reference parity: worker/zstep_worker/sampler.py:62 (SlotPenaltyState), :127
// (sample_tp8_logits: penalties, temperature, top-k, top-p, SplitMix64 uniform draw).
#include "sm100_common.cuh"
#include "zs_kernels.h"

namespace zs {
namespace smp {

constexpr int T = 1024;
constexpr int kHist = 4096;   // history tokens considered per row
constexpr int kTopN = 5;

ZS_DEVICE uint32_t okey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Deterministic block sum (fixed tree) of one value per thread.
ZS_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = red[threadIdx.x];
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

ZS_DEVICE unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffff, v, o);
    v = x > v ? x : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long t = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long x = __shfl_xor_sync(0xffffffff, t, o);
      t = x > t ? x : t;
    }
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const unsigned long long r = red[0];
  __syncthreads();
  return r;
}

ZS_DEVICE float uniform01(unsigned long long seed) {
  unsigned long long z = seed + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(T) sample_kernel(SampleArgs a) {
  pdl_wait();  // predecessor kernel done: its outputs are visible
  pdl_trigger();
  const int row = blockIdx.x, tid = threadIdx.x;
  const int V = a.vocab;
  float* lg = a.logits + (size_t)row * a.ld;
  __shared__ float red[32];
  __shared__ unsigned long long redu[32];
  __shared__ int hist_s[kHist];
  __shared__ float raw_h[kHist];  // raw logit of each distinct history token (at its first index)
  __shared__ float part[16][32];
  __shared__ uint32_t pick_s;
  // Contiguous token chunk of this thread (fixed-order reductions).
  const int chunk = (V + T - 1) / T;
  const int c0 = min(V, tid * chunk), c1 = min(V, c0 + chunk);

  // ---- raw log-probabilities (before penalties): log-sum-exp and top-N
  float lse = 0.f;
  if (a.want_logprobs) {
    float mx = -INFINITY;
    for (int i = c0; i < c1; ++i) mx = fmaxf(mx, lg[i]);
    const unsigned long long mk = block_max_u64((unsigned long long)okey(mx) << 32, redu);
    const uint32_t mb = (uint32_t)(mk >> 32);
    const float m = __uint_as_float((mb & 0x80000000u) ? (mb & 0x7FFFFFFFu) : ~mb);
    float se = 0.f;
    for (int i = c0; i < c1; ++i) se += expf(lg[i] - m);
    lse = m + logf(block_sum(se, red));
    // top-N by repeated block argmax over the not-yet-taken tokens
    int taken[kTopN];
    for (int n = 0; n < a.top_n && n < kTopN; ++n) {
      unsigned long long best = 0;
      for (int i = c0; i < c1; ++i) {
        bool used = false;
        for (int q = 0; q < n; ++q) used |= taken[q] == i;
        if (used) continue;
        const unsigned long long k = ((unsigned long long)okey(lg[i]) << 32) | (uint32_t)~(uint32_t)i;
        best = k > best ? k : best;
      }
      best = block_max_u64(best, redu);
      const int id = (int)~(uint32_t)(best & 0xFFFFFFFFu);
      taken[n] = id;
      if (tid == 0) {
        a.out_top_ids[row * kTopN + n] = id;
        a.out_top_lp[row * kTopN + n] = lg[id] - lse;
      }
    }
  }

  // ---- penalties, applied once per distinct history token
  const float pres = a.presence ? a.presence[row] : 0.f;
  const float freq = a.frequency ? a.frequency[row] : 0.f;
  const float rep = a.repetition ? a.repetition[row] : 1.f;
  const int hn = a.hist_len ? min(a.hist_len[row], kHist) : 0;
  const bool penalized = hn > 0 && (pres != 0.f || freq != 0.f || rep != 1.f);
  if (penalized) {
    for (int i = tid; i < kHist; i += T) hist_s[i] = i < hn ? a.hist[(size_t)row * a.hist_ld + i] : 0x7FFFFFFF;
    __syncthreads();
    for (int k = 2; k <= kHist; k <<= 1)  // bitonic sort, ascending
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < kHist; i += T) {
          const int l = i ^ j;
          if (l > i) {
            const int x = hist_s[i], y = hist_s[l];
            if (((i & k) == 0) == (x > y)) {
              hist_s[i] = y;
              hist_s[l] = x;
            }
          }
        }
        __syncthreads();
      }
    for (int i = tid; i < hn; i += T) {
      const int t = hist_s[i];
      if ((i == 0 || hist_s[i - 1] != t) && t >= 0 && t < V) {
        int cnt = 1;
        while (i + cnt < hn && hist_s[i + cnt] == t) ++cnt;
        float v = lg[t];
        raw_h[i] = v;
        if (rep != 1.f) v = v > 0.f ? v / rep : v * rep;
        lg[t] = v - freq * (float)cnt - pres;
      }
    }
    __syncthreads();
  }

  const float temp = a.temperature[row];
  int token = 0;
  if (!(temp > 0.f)) {
    unsigned long long best = 0;
    for (int i = c0; i < c1; ++i) {
      const unsigned long long k = ((unsigned long long)okey(lg[i]) << 32) | (uint32_t)~(uint32_t)i;
      best = k > best ? k : best;
    }
    best = block_max_u64(best, redu);
    token = (int)~(uint32_t)(best & 0xFFFFFFFFu);
  } else {
    const float inv_t = 1.f / temp;
    // max of s = l / T
    float mx = -INFINITY;
    for (int i = c0; i < c1; ++i) mx = fmaxf(mx, lg[i]);
    const unsigned long long mk = block_max_u64((unsigned long long)okey(mx) << 32, redu);
    const uint32_t mb = (uint32_t)(mk >> 32);
    const float m = __uint_as_float((mb & 0x80000000u) ? (mb & 0x7FFFFFFFu) : ~mb) * inv_t;
    // top-k threshold key (0: keep everything)
    uint32_t kthr = 0;
    const int K = a.top_k ? a.top_k[row] : 0;
    if (K > 0 && K < V) {
      uint32_t prefix = 0;
      int need = K;
      for (int pass = 0; pass < 8; ++pass) {
        const int shift = 28 - 4 * pass;
        const uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 4 * pass));
        int cnt[16];
#pragma unroll
        for (int d = 0; d < 16; ++d) cnt[d] = 0;
        for (int i = c0; i < c1; ++i) {
          const uint32_t k = okey(lg[i] * inv_t);
          if ((k & pmask) == prefix) ++cnt[(k >> shift) & 15];
        }
        __syncthreads();
#pragma unroll
        for (int d = 0; d < 16; ++d) {
          const float v = warp_sum((float)cnt[d]);
          if ((tid & 31) == 0) part[d][tid >> 5] = v;
        }
        __syncthreads();
        if (tid == 0) {
          int d = 15;
          for (; d > 0; --d) {
            float c = 0.f;
            for (int w = 0; w < 32; ++w) c += part[d][w];
            if ((int)c >= need) break;
            need -= (int)c;
          }
          pick_s = prefix | ((uint32_t)d << shift);
        }
        __syncthreads();
        prefix = pick_s;
      }
      kthr = prefix;
    }
    // mass of the top-k set and the top-p threshold key
    auto kept_k = [&](uint32_t k) { return k >= kthr; };
    float zs = 0.f;
    for (int i = c0; i < c1; ++i) {
      const float s = lg[i] * inv_t;
      if (kept_k(okey(s))) zs += expf(s - m);
    }
    const float zk = block_sum(zs, red);
    uint32_t pthr = kthr;
    const float P = a.top_p ? a.top_p[row] : 1.f;
    if (P < 1.f) {
      const float target = P * zk;
      uint32_t prefix = 0;
      float above = 0.f;  // mass of keys above the current prefix range
      for (int pass = 0; pass < 8; ++pass) {
        const int shift = 28 - 4 * pass;
        const uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 4 * pass));
        float ms[16];
#pragma unroll
        for (int d = 0; d < 16; ++d) ms[d] = 0.f;
        for (int i = c0; i < c1; ++i) {
          const float s = lg[i] * inv_t;
          const uint32_t k = okey(s);
          if (kept_k(k) && (k & pmask) == prefix) ms[(k >> shift) & 15] += expf(s - m);
        }
        __syncthreads();
#pragma unroll
        for (int d = 0; d < 16; ++d) {
          const float v = warp_sum(ms[d]);
          if ((tid & 31) == 0) part[d][tid >> 5] = v;
        }
        __syncthreads();
        if (tid == 0) {
          float run = above;
          int d = 15;
          for (; d > 0; --d) {
            float c = 0.f;
            for (int w = 0; w < 32; ++w) c += part[d][w];
            if (run + c >= target) break;
            run += c;
          }
          pick_s = prefix | ((uint32_t)d << shift);
          red[0] = run;
        }
        __syncthreads();
        prefix = pick_s;
        above = red[0];
        __syncthreads();
      }
      pthr = prefix > kthr ? prefix : kthr;
    }
    // draw: kept mass in token-id order
    float mine = 0.f;
    for (int i = c0; i < c1; ++i) {
      const float s = lg[i] * inv_t;
      if (okey(s) >= pthr) mine += expf(s - m);
    }
    // exclusive scan of the per-thread masses (fixed order)
    __shared__ float scan[T];
    scan[tid] = mine;
    __syncthreads();
    for (int off = 1; off < T; off <<= 1) {
      const float v = tid >= off ? scan[tid - off] : 0.f;
      __syncthreads();
      scan[tid] += v;
      __syncthreads();
    }
    const float total = scan[T - 1];
    const float goal = uniform01(a.seed[row]) * total;
    const float before = scan[tid] - mine;
    if (tid == 0) pick_s = 0xFFFFFFFFu;
    __syncthreads();
    if (mine > 0.f && goal >= before && goal < before + mine) {
      float run = before;
      int pick = -1, last = -1;
      for (int i = c0; i < c1; ++i) {
        const float s = lg[i] * inv_t;
        if (okey(s) < pthr) continue;
        last = i;
        run += expf(s - m);
        if (goal < run) {
          pick = i;
          break;
        }
      }
      atomicMin(&pick_s, (uint32_t)(pick >= 0 ? pick : last));
    }
    __syncthreads();
    if (pick_s == 0xFFFFFFFFu) {  // rounding at the very end of the mass: last kept token
      unsigned long long best = 0;
      for (int i = c0; i < c1; ++i)
        if (okey(lg[i] * inv_t) >= pthr) best = (unsigned long long)(i + 1) > best ? (unsigned long long)(i + 1) : best;
      best = block_max_u64(best, redu);
      token = (int)best - 1;
    } else {
      token = (int)pick_s;
    }
  }
  if (tid == 0) {
    a.out_token[row] = token;
    if (a.want_logprobs) {
      float raw = lg[token];
      if (penalized) {  // the chosen token may have been penalised in place: use its saved raw logit
        int lo = 0, hi = hn;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (hist_s[mid] < token) lo = mid + 1; else hi = mid;
        }
        if (lo < hn && hist_s[lo] == token) raw = raw_h[lo];
      }
      a.out_logprob[row] = raw - lse;
    }
  }
}

}  // namespace smp
}  // namespace zs

extern "C" int zs_sample(const SampleArgs* args, cudaStream_t stream) {
  const SampleArgs& a = *args;
  if (a.rows <= 0) return 0;
  if (a.vocab <= 0 || a.ld < a.vocab || a.top_n > zs::smp::kTopN || a.hist_ld > 0 && a.hist == nullptr) return -1;
  zs_launch(zs::smp::sample_kernel, a.rows, zs::smp::T, 0, stream, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------------------------------
// On-device greedy verify of a speculative step (one CTA, one thread per sequence).
//
// Sequence i owns rows [i*(K+1), (i+1)*(K+1)): its last accepted token then K drafts.
// targets[row] is the target model's greedy token after that row.  The accepted prefix is
// the longest run j = 0.. with targets[i*(K+1)+j] == ids[i*(K+1)+j+1], plus the target token
// that follows it (the bonus), so 1 <= acc_len <= K+1 and the accepted tokens are
// targets[i*(K+1) .. i*(K+1)+acc_len).  The kernel also lays out what the rest of the step
// needs, all on the device:
//   * the recurrent-state replay over the accepted rows: a compacted row list with its
//     per-sequence starts (an exclusive prefix sum of acc_len), slots and positions;
//   * the draft head's catch-up rows (fixed size n*(K+1): row j of sequence i carries the
//     token that followed it if j < acc_len, else points at the padding slot);
//   * the catch-up row of each sequence's newest token (where the next drafts start);
//   * the host-visible record: acc_len then the K+1 token slots (-1 past acc_len).
// Reference parity: worker/zstep_worker/spec_decode.py:41 (verify_greedy), :55 (verify_batch).
namespace zs {
__global__ void __launch_bounds__(1024) spec_verify_kernel(const SpecVerifyArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ int scan[1024];
  const int i = threadIdx.x, K1 = a.k + 1;
  int acc = 0;
  if (i < a.n) {
    const int r0 = i * K1;
    acc = 1;
    while (acc < K1 && a.targets[r0 + acc - 1] == a.ids[r0 + acc]) ++acc;
    int* rec = a.record + (size_t)i * (K1 + 1);
    rec[0] = acc;
    for (int j = 0; j < K1; ++j) {
      const int r = r0 + j;
      const bool ok = j < acc;
      rec[1 + j] = ok ? a.targets[r] : -1;
      a.mtp_ids[r] = ok ? a.targets[r] : 0;
      a.mtp_pos[r] = ok ? a.pos[r] : 1;
      a.mtp_slot[r] = ok ? a.slot[r] : a.dummy_slot;
      a.mtp_len[r] = ok ? a.pos[r] + 1 : 2;
    }
    a.last_row[i] = r0 + acc - 1;
  }
  // Exclusive prefix sum of acc over the sequences (Hillis-Steele in shared memory).
  scan[i] = acc;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    const int v = i >= off ? scan[i - off] : 0;
    __syncthreads();
    scan[i] += v;
    __syncthreads();
  }
  if (i < a.n) {
    const int start = scan[i] - acc;
    a.rep_start[i] = start;
    if (i == a.n - 1) a.rep_start[a.n] = scan[i];
    const int r0 = i * K1;
    for (int j = 0; j < acc; ++j) {
      a.rep_idx[start + j] = r0 + j;
      a.rep_slot[start + j] = a.slot[r0];
      a.rep_pos[start + j] = a.pos[r0 + j];
    }
  }
}
}  // namespace zs

extern "C" int zs_spec_verify(const SpecVerifyArgs* args, cudaStream_t stream) {
  const SpecVerifyArgs& a = *args;
  if (a.n < 1 || a.n > 1024 || a.k < 1 || a.k > 7) return -1;
  return zs_launch(zs::spec_verify_kernel, 1, 1024, 0, stream, a) == cudaSuccess &&
                 cudaGetLastError() == cudaSuccess
             ? 0
             : -2;
}

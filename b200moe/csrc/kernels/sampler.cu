// Token sampler (sm_100a).  One CTA of 1024 threads per row of fp32 logits.
//
//   greedy rows          argmax, lowest token id on ties
//   sampled rows         logits / temperature -> top-k -> top-p -> min-p ->
//                        exponential race: argmax_i p_i / E_i with E_i ~ Exp(1)
//                        (the reference's sampler, nanovllm/layers/sampler.py:112-169,
//                        which sorts the whole vocabulary for top-k / top-p)
//   guided rows          an allowed-token bitmask removes tokens before all of the above
//   log-probs            of the distribution the row samples from (temperature and
//                        filters applied; greedy rows: the raw logits), the chosen
//                        token's and the top lp_k (<= 20) -- reference semantics of
//                        nanovllm/layers/sampler.py:_gather_logprobs
//
// No sort: the top-k and top-p thresholds come from an MSB-first radix select
// over the order-preserving integer image of the scaled logits (4 passes of 8
// bits; top-k counts tokens per bucket, top-p accumulates probability mass per
// bucket).  Ties at the threshold are kept.  Random numbers come from the
// Philox-4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw:
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011), keyed by the row's
// seed and counted by (token id, step offset), so a row's draw does not depend
// on the batch it runs in.
//
// Penalties (repetition on prompt+generated, presence / frequency on
// generated ids) are applied in place by a separate kernel before sampling.
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sm100.cuh"
#include "pdl.cuh"
#include "sampler.h"

namespace b200 {

constexpr int kST = 1024;

__device__ __forceinline__ uint32_t f2ord(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Philox 4x32, 10 rounds (multipliers and Weyl keys from the SC'11 paper).
__device__ __forceinline__ uint4 philox4x32(uint4 ctr, uint2 key) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
    const uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += W0;
    key.y += W1;
  }
  return ctr;
}

// uniform in (0, 1]
__device__ __forceinline__ float u01(uint32_t x) { return (float)((x >> 8) + 1) * (1.0f / 16777216.0f); }

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float s = l < kST / 32 ? red[l] : 0.f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (l == 0) red[0] = s;
  }
  __syncthreads();
  const float s = red[0];
  __syncthreads();
  return s;
}

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float s = l < kST / 32 ? red[l] : -INFINITY;
    for (int o = 16; o > 0; o >>= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (l == 0) red[0] = s;
  }
  __syncthreads();
  const float s = red[0];
  __syncthreads();
  return s;
}

// (value, index) argmax with lowest index on ties
__device__ __forceinline__ void block_argmax(float& v, int& idx, float* redv, int* redi) {
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) { redv[w] = v; redi[w] = idx; }
  __syncthreads();
  if (w == 0) {
    v = l < kST / 32 ? redv[l] : -INFINITY;
    idx = l < kST / 32 ? redi[l] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
    if (l == 0) { redv[0] = v; redi[0] = idx; }
  }
  __syncthreads();
  v = redv[0];
  idx = redi[0];
  __syncthreads();
}

__global__ void __launch_bounds__(kST) argmax_kernel(const float* __restrict__ logits, int V, int64_t ld,
                                                     int* __restrict__ out) {
  pdl_enter();
  __shared__ float redv[32];
  __shared__ int redi[32];
  const float* row = logits + (size_t)blockIdx.x * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += kST) {
    const float v = row[i];
    if (v > bv) { bv = v; bi = i; }  // strided scan: first hit per thread is its lowest index
  }
  block_argmax(bv, bi, redv, redi);
  if (threadIdx.x == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  pdl_trigger();
}

// Token i passes the allowed-token bitmask (null mask: every token does).
__device__ __forceinline__ bool allowed(const uint32_t* am, int i) {
  return am == nullptr || ((am[i >> 5] >> (i & 31)) & 1u);
}

// Radix select over the ordered image of x/temp among allowed tokens with image >= lo_bound.
// mode 0: image of the k-th largest value (k counted from the top)
// mode 1: largest image t such that the probability mass of tokens with image
//         >= t reaches `target` (mass weight exp(x - M) * invZ)

__device__ uint32_t radix_select(const float* row, int V, float inv_t, uint32_t lo_bound, int mode, int k,
                                 float target, float M, float invZ, const uint32_t* am, uint32_t* hist_u,
                                 float* hist_f) {
  uint32_t prefix = 0, mask = 0;
  float above_mass = 0.f;
  uint32_t above_cnt = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kST) { hist_u[i] = 0; hist_f[i] = 0.f; }
    __syncthreads();
    if (mode == 0) {
      for (int i = threadIdx.x; i < V; i += kST) {
        if (!allowed(am, i)) continue;
        const uint32_t o = f2ord(row[i] * inv_t);
        if (o < lo_bound || (o & mask) != prefix) continue;
        atomicAdd(&hist_u[(o >> shift) & 0xFFu], 1u);
      }
    } else {
      // Probability mass: logits of a row share a few exponents, so the high digits put
      // most values in one or two bins, and fp32 shared-memory atomics on one address
      // serialise.  Each thread keeps two (bin, mass) accumulators in registers; values of
      // a third bin go to the atomics directly, the accumulators join once at the end.
      // (Counts keep the plain atomics: measured faster there.)
      uint32_t ba = 0xFFFFFFFFu, bb = 0xFFFFFFFFu;
      float ma = 0.f, mb = 0.f;
      for (int i = threadIdx.x; i < V; i += kST) {
        if (!allowed(am, i)) continue;
        const float x = row[i] * inv_t;
        const uint32_t o = f2ord(x);
        if (o < lo_bound || (o & mask) != prefix) continue;
        const uint32_t bin = (o >> shift) & 0xFFu;
        const float v = __expf(x - M) * invZ;
        if (bin == ba) ma += v;
        else if (bin == bb) mb += v;
        else if (ba == 0xFFFFFFFFu) { ba = bin; ma = v; }
        else if (bb == 0xFFFFFFFFu) { bb = bin; mb = v; }
        else atomicAdd(&hist_f[bin], v);
      }
      if (ba != 0xFFFFFFFFu) atomicAdd(&hist_f[ba], ma);
      if (bb != 0xFFFFFFFFu) atomicAdd(&hist_f[bb], mb);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int l = threadIdx.x;
      // each lane owns 8 bins, lane 0 the highest
      float m8[8];
      uint32_t c8[8];
      float ms = 0.f;
      uint32_t cs = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int bin = 255 - (l * 8 + j);
        m8[j] = hist_f[bin];
        c8[j] = hist_u[bin];
        ms += m8[j];
        cs += c8[j];
      }
      float mi = ms;
      uint32_t ci = cs;
      for (int o = 1; o < 32; o <<= 1) {
        const float mv = __shfl_up_sync(0xffffffffu, mi, o);
        const uint32_t cv = __shfl_up_sync(0xffffffffu, ci, o);
        if (l >= o) { mi += mv; ci += cv; }
      }
      float mpre = mi - ms;
      uint32_t cpre = ci - cs;
      int found = -1;
      float m_before = 0.f;
      uint32_t c_before = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool hit = mode == 0 ? (above_cnt + cpre + c8[j] >= (uint32_t)k)
                                   : (above_mass + mpre + m8[j] >= target);
        if (found < 0 && hit) { found = 255 - (l * 8 + j); m_before = mpre; c_before = cpre; }
        mpre += m8[j];
        cpre += c8[j];
      }
      const unsigned ball = __ballot_sync(0xffffffffu, found >= 0);
      const int src = ball ? __ffs(ball) - 1 : 31;
      const int fbin = __shfl_sync(0xffffffffu, found, src);
      const float mb = __shfl_sync(0xffffffffu, m_before, src);
      const uint32_t cb = __shfl_sync(0xffffffffu, c_before, src);
      if (l == 0) {
        hist_u[256] = ball ? (uint32_t)fbin : 0u;
        hist_f[256] = ball ? mb : 0.f;
        hist_u[257] = ball ? cb : 0u;
      }
    }
    __syncthreads();
    const uint32_t bin = hist_u[256];
    above_mass += hist_f[256];
    above_cnt += hist_u[257];
    prefix |= bin << shift;
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  return prefix;
}

constexpr int kCand = 64;  // candidates gathered for the top log-probs (ties past it are dropped)
constexpr int kCompact = 1024;  // top-k survivors kept in shared memory for the rest of a row's sampling

// The k best (value, id) among allowed tokens whose scaled image is >= lo, best
// first (ties: lower id first), written as log-probabilities x - M - logZ.
__device__ void write_top_logprobs(const float* row, int V, float inv_t, uint32_t lo, const uint32_t* am, int k,
                                   float M, float logZ, uint32_t* hist_u, float* hist_f, float* cv, int* ci,
                                   int* nc, float* out_v, int* out_i) {
  const uint32_t t = radix_select(row, V, inv_t, lo, 0, k, 0.f, M, 1.f, am, hist_u, hist_f);
  const uint32_t bound = max(t, lo);
  if (threadIdx.x == 0) *nc = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += kST) {
    if (!allowed(am, i)) continue;
    const float x = row[i] * inv_t;
    if (f2ord(x) < bound) continue;
    const int slot = atomicAdd(nc, 1);
    if (slot < kCand) { cv[slot] = x; ci[slot] = i; }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int n = min(*nc, kCand);
    for (int p = 1; p < n; ++p) {  // insertion sort of <= 64 entries
      const float v = cv[p];
      const int id = ci[p];
      int q = p - 1;
      while (q >= 0 && (cv[q] < v || (cv[q] == v && ci[q] > id))) {
        cv[q + 1] = cv[q];
        ci[q + 1] = ci[q];
        --q;
      }
      cv[q + 1] = v;
      ci[q + 1] = id;
    }
    for (int j = 0; j < k; ++j) {
      out_v[j] = j < n ? cv[j] - M - logZ : -INFINITY;
      out_i[j] = j < n ? ci[j] : -1;
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kST) sample_kernel(const float* __restrict__ logits, int V, int64_t ld,
                                                     SampleArgs a, int* __restrict__ out) {
  pdl_enter();
  __shared__ float red[32];
  __shared__ int redi[32];
  __shared__ uint32_t hist_u[260];
  __shared__ float hist_f[260];
  __shared__ float cand_v[kCand];
  __shared__ int cand_i[kCand];
  __shared__ int n_cand;
  __shared__ float comp_x[kCompact];
  __shared__ int comp_i[kCompact];
  __shared__ int n_comp;
  const int r = blockIdx.x;
  const float* row = logits + (size_t)r * ld;
  const uint32_t* am = nullptr;
  if (a.allow != nullptr && a.allow_row != nullptr && a.allow_row[r] >= 0)
    am = a.allow + (size_t)a.allow_row[r] * a.mask_words;
  const float temp = a.temperature[r];
  const bool greedy = temp < 1e-3f;
  const float inv_t = greedy ? 1.f : 1.f / temp;
  const int lp_k = a.lp_k;

  // best allowed token of the scaled logits: the greedy choice and the softmax max
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += kST) {
    if (!allowed(am, i)) continue;
    const float x = row[i] * inv_t;
    if (x > bv) { bv = x; bi = i; }  // strided scan: first hit per thread is its lowest index
  }
  block_argmax(bv, bi, red, redi);
  const float M = bv;
  if (M == -INFINITY) {  // nothing allowed (or every logit -inf): token 0, no distribution
    if (threadIdx.x == 0) out[r] = 0;
    if (lp_k > 0 && threadIdx.x < lp_k) {
      a.lp_top_v[(size_t)r * lp_k + threadIdx.x] = -INFINITY;
      a.lp_top_i[(size_t)r * lp_k + threadIdx.x] = -1;
    }
    if (lp_k > 0 && threadIdx.x == 0) a.lp_chosen[r] = -INFINITY;
    return;
  }

  uint32_t lo = 0;  // the distribution: allowed tokens with f2ord(x) >= lo
  int tok;
  // top-k survivors (scaled logits and ids) compacted into shared memory when they fit:
  // the nucleus, the min-p bound, the draw and the sampled distribution's normaliser
  // then walk at most kCompact entries instead of the whole row
  int nc = -1;  // -1: not compacted
  if (greedy) {
    tok = bi;
  } else {
    const int top_k = a.top_k ? a.top_k[r] : -1;
    if (top_k > 0 && top_k < V) {
      lo = radix_select(row, V, inv_t, 0, 0, top_k, 0.f, M, 1.f, am, hist_u, hist_f);
      if (top_k <= kCompact) {
        if (threadIdx.x == 0) n_comp = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < V; i += kST) {
          if (!allowed(am, i)) continue;
          const float x = row[i] * inv_t;
          if (f2ord(x) < lo) continue;
          const int slot = atomicAdd(&n_comp, 1);
          if (slot < kCompact) { comp_x[slot] = x; comp_i[slot] = i; }
        }
        __syncthreads();
        nc = n_comp <= kCompact ? n_comp : -1;  // ties past the cap: the whole row again
        __syncthreads();
      }
    }
    const float top_p = a.top_p ? a.top_p[r] : 1.f;
    if (top_p < 1.f) {
      // nucleus mass is measured over the top-k survivors
      float zk = 0.f;
      if (nc >= 0) {
        for (int j = threadIdx.x; j < nc; j += kST) zk += __expf(comp_x[j] - M);
      } else {
        for (int i = threadIdx.x; i < V; i += kST) {
          if (!allowed(am, i)) continue;
          const float x = row[i] * inv_t;
          if (f2ord(x) >= lo) zk += __expf(x - M);
        }
      }
      const float Zk = block_reduce_sum(zk, red);
      const uint32_t tp = nc >= 0 ? radix_select(comp_x, nc, 1.f, lo, 1, 0, top_p, M, 1.f / Zk, nullptr, hist_u, hist_f)
                                  : radix_select(row, V, inv_t, lo, 1, 0, top_p, M, 1.f / Zk, am, hist_u, hist_f);
      lo = max(lo, tp);
    }
    const float min_p = a.min_p ? a.min_p[r] : 0.f;
    if (min_p > 0.f) lo = max(lo, f2ord(M + __logf(min_p)));

    const uint2 key = make_uint2((uint32_t)a.seeds[r], (uint32_t)((uint64_t)a.seeds[r] >> 32));
    const uint32_t off = a.offsets ? (uint32_t)a.offsets[r] : 0u;
    float sv = -INFINITY;
    int si = 0x7fffffff;
    // exponential race keyed by the token id: the same draw whether or not the
    // survivors were compacted
    auto race = [&](int i, float x) {
      if (f2ord(x) < lo) return;
      const uint4 rnd = philox4x32(make_uint4((uint32_t)i, off, 0x5A3Cu, 0u), key);
      const float e = -__logf(u01(rnd.x));  // Exp(1)
      const float score = (x - M) - __logf(fmaxf(e, 1e-20f));
      if (score > sv || (score == sv && i < si)) { sv = score; si = i; }
    };
    if (nc >= 0) {
      for (int j = threadIdx.x; j < nc; j += kST) race(comp_i[j], comp_x[j]);
    } else {
      for (int i = threadIdx.x; i < V; i += kST)
        if (allowed(am, i)) race(i, row[i] * inv_t);
    }
    block_argmax(sv, si, red, redi);
    tok = si == 0x7fffffff ? bi : si;
  }
  if (threadIdx.x == 0) out[r] = tok;
  if (lp_k <= 0) return;

  // log-probabilities of the distribution just sampled from
  float zs = 0.f;
  if (nc >= 0) {
    for (int j = threadIdx.x; j < nc; j += kST)
      if (f2ord(comp_x[j]) >= lo) zs += expf(comp_x[j] - M);
  } else {
    for (int i = threadIdx.x; i < V; i += kST) {
      if (!allowed(am, i)) continue;
      const float x = row[i] * inv_t;
      if (f2ord(x) >= lo) zs += expf(x - M);
    }
  }
  const float logZ = logf(block_reduce_sum(zs, red));
  if (threadIdx.x == 0) a.lp_chosen[r] = row[tok] * inv_t - M - logZ;
  write_top_logprobs(row, V, inv_t, lo, am, lp_k, M, logZ, hist_u, hist_f, cand_v, cand_i, &n_cand,
                     a.lp_top_v + (size_t)r * lp_k, a.lp_top_i + (size_t)r * lp_k);
  pdl_trigger();
}

__global__ void penalty_kernel(float* __restrict__ logits, int64_t ld, const int* __restrict__ rows,
                               const int* __restrict__ ids, const int* __restrict__ gen_counts,
                               const float* __restrict__ presence, const float* __restrict__ frequency,
                               const float* __restrict__ repetition, int n) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = rows[i];
  float* p = logits + (size_t)r * ld + ids[i];
  float v = *p;
  const float rp = repetition[r];
  v = v < 0.f ? v * rp : v / rp;
  const int c = gen_counts[i];
  if (c > 0) v = v - presence[r] - frequency[r] * (float)c;
  *p = v;
  pdl_trigger();
}

static void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void argmax_rows(const float* logits, int B, int V, int64_t ld, int* out, cudaStream_t s) {
  if (B == 0) return;
  pdl_launch(argmax_kernel, B, kST, 0, s, logits, V, ld, out);
  check_launch("argmax_rows");
}

void sample_rows(const float* logits, int B, int V, int64_t ld, const SampleArgs& a, int* out, cudaStream_t s) {
  if (B == 0) return;
  if (a.lp_k < 0 || a.lp_k > kMaxLogprobs) throw std::runtime_error("sample_rows: lp_k out of [0, 20]");
  if (a.lp_k > 0 && (a.lp_top_v == nullptr || a.lp_top_i == nullptr || a.lp_chosen == nullptr))
    throw std::runtime_error("sample_rows: log-prob outputs missing");
  if ((a.allow == nullptr) != (a.allow_row == nullptr) || (a.allow != nullptr && a.mask_words * 32 < V))
    throw std::runtime_error("sample_rows: allowed-token mask needs both arrays and ceil(V / 32) words");
  pdl_launch(sample_kernel, B, kST, 0, s, logits, V, ld, a, out);
  check_launch("sample_rows");
}

void apply_penalties(float* logits, int64_t ld, const int* rows, const int* ids, const int* gen_counts,
                     const float* presence, const float* frequency, const float* repetition, int n,
                     cudaStream_t s) {
  if (n == 0) return;
  pdl_launch(penalty_kernel, (n + 255) / 256, 256, 0, s, logits, ld, rows, ids, gen_counts, presence, frequency,
                                                 repetition, n);
  check_launch("apply_penalties");
}

}  // namespace b200

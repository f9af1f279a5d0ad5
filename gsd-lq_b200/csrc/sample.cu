// sample.cu -- temperature + top-p sampling on the device: the rules of the reference's sample_token
// (gsd_lq_cpu_runtime.py:422-443), one CTA per call, so that a sampled decode loop needs no host round
// trip per token.
//
// The reference: logits with NaN -> -1e4, +inf -> 100, -inf -> -1e4; greedy argmax when T <= 0;
// z = logits / max(T, 1e-4) (fp32); z -= max z; e = exp(z); s = sum e (argmax when s <= 0 or NaN);
// p = e / s; p sorted descending; the nucleus is the first k entries, k = 1 + the first index whose
// running sum exceeds top_p (k = 1 when none does); P = sum of the nucleus (its first entry when P <= 0
// or NaN); np.random.choice over the nucleus with p / P takes the first entry whose running float64
// sum, divided by the total, exceeds the uniform draw u.
//
// Here the sorted order is never built.  Both "first entry in descending order of p whose running sum
// exceeds a target" questions are answered by a radix select over p's float bits (non-negative floats
// order as their bit patterns), most significant byte first: a 256-bucket histogram of counts and of
// mass (exact 2^-56 fixed point, so that the sums do not depend on the order of the atomics) locates the
// bucket in which the running mass crosses the target, four times, which leaves the exact value v at the
// crossing; entries equal to v are taken in ascending index order (the reference's order among equal
// probabilities is that of NumPy's argsort, which is unspecified) and the crossing one is the t-th of
// them.  The running sums are exact here and rounded float32 / float64 sums in the reference, so a pick
// can differ from the reference's where the target lies within rounding distance of a running sum
// (top_p = 1 is such a case: whether the reference's float32 running sum ever exceeds 1 depends on its
// rounding), and where the reference's exp differs from CUDA's in the last bit at such a boundary.
#include <cmath>
#include <cstdint>

#include "common.cuh"

namespace gsdlq {

constexpr int SMP_THREADS = 1024;
constexpr double SMP_ONE = 72057594037927936.0;  // 2^56: the fixed-point unit of probability mass

__device__ __forceinline__ float smp_clean(float l) {  // np.nan_to_num(l, nan=-1e4, posinf=100, neginf=-1e4)
  if (isnan(l)) return -1e4f;
  if (isinf(l)) return l > 0.f ? 100.f : -1e4f;
  return l;
}
__device__ __forceinline__ unsigned long long smp_fix(float p) {
  return (unsigned long long)((double)p * SMP_ONE);  // p in [0, 1]: exact to 2^-56
}

struct SmpShared {
  unsigned int cnt[256];
  unsigned long long mass[256];
  unsigned long long ured[32];
  unsigned int ired[32];
  float fred[32];
  int ibest[32];
  uint32_t prefix;
  unsigned long long mass_above;
  int found, index;
};

__device__ float smp_block_max(SmpShared& S, float v) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) S.fred[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = S.fred[l];
    t = warp_max(t);
    if (l == 0) S.fred[0] = t;
  }
  __syncthreads();
  return S.fred[0];
}
__device__ float smp_block_sum(SmpShared& S, float v) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) S.fred[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = S.fred[l];
    t = warp_sum(t);
    if (l == 0) S.fred[0] = t;
  }
  __syncthreads();
  return S.fred[0];
}
__device__ unsigned long long smp_block_sum_u64(SmpShared& S, unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) S.ured[w] = v;
  __syncthreads();
  if (w == 0) {
    unsigned long long t = S.ured[l];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) S.ured[0] = t;
  }
  __syncthreads();
  return S.ured[0];
}
// the lowest index i with key(i) = the maximum key among members (-1 when there is no member)
template <class KEY, class MEMBER>
__device__ int smp_first_max(SmpShared& S, int n, KEY key, MEMBER member) {
  uint32_t best = 0u;
  int bi = -1;
  for (int i = threadIdx.x; i < n; i += SMP_THREADS) {
    if (!member(i)) continue;
    const uint32_t k = key(i);
    if (bi < 0 || k > best) best = k, bi = i;  // i ascends within a thread
  }
  // (key, ~index) order: the larger key, then the smaller index
  unsigned long long v = bi < 0 ? 0ull : (((unsigned long long)best << 32) | (0xffffffffu - (uint32_t)bi));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) S.ured[w] = v;
  __syncthreads();
  if (w == 0) {
    unsigned long long t = S.ured[l];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long u = __shfl_xor_sync(0xffffffffu, t, o);
      t = u > t ? u : t;
    }
    if (l == 0) S.ured[0] = t;
  }
  __syncthreads();
  const unsigned long long r = S.ured[0];
  __syncthreads();
  return r == 0ull ? -1 : (int)(0xffffffffu - (uint32_t)(r & 0xffffffffull));
}

// The first entry, in descending order of key (ties by ascending index), at which the running sum of
// mass over the member entries exceeds `target`.  Returns its index, or -1 when the whole sum does not
// exceed the target.
template <class KEY, class MASS, class MEMBER>
__device__ int smp_select(SmpShared& S, int n, unsigned long long target, KEY key, MASS mass, MEMBER member) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid == 0) {
    S.prefix = 0u;
    S.mass_above = 0ull;
  }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t hi_mask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
    for (int b = tid; b < 256; b += SMP_THREADS) {
      S.cnt[b] = 0u;
      S.mass[b] = 0ull;
    }
    __syncthreads();
    const uint32_t prefix = S.prefix;
    for (int base = 0; base < n; base += SMP_THREADS) {  // every lane takes part in every round
      const int i = base + tid;
      uint32_t bucket = 256u;
      unsigned long long m = 0ull;
      if (i < n && member(i)) {
        const uint32_t k = key(i);
        if ((k & hi_mask) == (prefix & hi_mask)) {
          bucket = (k >> shift) & 0xffu;
          m = mass(i);
        }
      }
      // warp-aggregated update: the lanes of one bucket sum their masses (three 21-bit pieces, so that
      // the 32-bit reductions cannot overflow) and one of them adds the sum
      const uint32_t peers = __match_any_sync(0xffffffffu, bucket);
      const unsigned long long m0 = __reduce_add_sync(peers, (unsigned)(m & 0x1fffffull));
      const unsigned long long m1 = __reduce_add_sync(peers, (unsigned)((m >> 21) & 0x1fffffull));
      const unsigned long long m2 = __reduce_add_sync(peers, (unsigned)(m >> 42));
      if (bucket < 256u && lane == __ffs(peers) - 1) {
        atomicAdd(&S.cnt[bucket], (unsigned)__popc(peers));
        atomicAdd(&S.mass[bucket], m0 + (m1 << 21) + (m2 << 42));
      }
    }
    __syncthreads();
    if (tid == 0) {  // the bucket, from the top, in which the running mass crosses the target
      unsigned long long cum = S.mass_above;
      int hit = -1;
      for (int b = 255; b >= 0; --b) {
        if (S.cnt[b] == 0u) continue;
        if (cum + S.mass[b] > target) {
          hit = b;
          break;
        }
        cum += S.mass[b];
      }
      S.found = hit >= 0;
      if (hit >= 0) {
        S.prefix = (prefix & hi_mask) | ((uint32_t)hit << shift);
        S.mass_above = cum;
      }
    }
    __syncthreads();
    if (!S.found) return -1;
  }
  // the entries of key v = prefix, in ascending index order, each of mass mv: the running sum crosses
  // at the t-th, t = floor((target - above) / mv) + 1
  const uint32_t kv = S.prefix;
  const unsigned long long above = S.mass_above;
  // each thread takes a contiguous range of indices, counts its entries of key v and finds mv
  const int chunk = (n + SMP_THREADS - 1) / SMP_THREADS;
  const int i0 = min(n, tid * chunk), i1 = min(n, i0 + chunk);
  unsigned c = 0u;
  unsigned long long mv = 0ull;
  for (int i = i0; i < i1; ++i)
    if (member(i) && key(i) == kv) {
      ++c;
      mv = mass(i);
    }
  // exclusive scan of the counts over the threads
  unsigned incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  const int w = tid >> 5;
  __syncthreads();
  if (lane == 31) S.ired[w] = incl;
  if (mv != 0ull) S.ured[0] = mv;  // every entry of key v has the same mass
  __syncthreads();
  if (w == 0) {
    unsigned t = S.ired[lane], ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned u = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += u;
    }
    S.ired[lane] = ti - t;  // exclusive prefix of the warps
  }
  __syncthreads();
  const unsigned excl = S.ired[w] + incl - c;
  const unsigned long long m_v = S.ured[0];
  const unsigned long long t =
      m_v == 0ull ? 1ull : (target >= above ? (target - above) / m_v : 0ull) + 1ull;  // 1-based
  if (tid == 0) S.index = -1;
  __syncthreads();
  if ((unsigned long long)excl < t && t <= (unsigned long long)(excl + c)) {
    unsigned need = (unsigned)(t - excl);
    for (int i = i0; i < i1; ++i)
      if (member(i) && key(i) == kv && --need == 0u) {
        S.index = i;
        break;
      }
  }
  __syncthreads();
  const int r = S.index;
  __syncthreads();
  return r;
}

// logits [n] -> *out_index; work: n floats (the probabilities); u: the draw (u_index >= 0: u[*u_index])
__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(const float* __restrict__ logits, int n, float temperature,
                                                             float top_p, const double* __restrict__ u,
                                                             const int* __restrict__ u_index, float* __restrict__ p,
                                                             unsigned long long* __restrict__ key_out,
                                                             int* __restrict__ index_out) {
  __shared__ SmpShared S;
  const int tid = threadIdx.x;
  auto all = [](int) { return true; };
  auto lkey = [&](int i) {  // order of the cleaned logits (for the greedy pick): monotone 32-bit map
    const uint32_t b = __float_as_uint(smp_clean(logits[i]));
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  };
  int pick = -1;
  if (!(temperature > 0.f)) {
    pick = smp_first_max(S, n, lkey, all);
  } else {
    const float tc = fmaxf(temperature, 1e-4f);
    float m = -INFINITY;
    for (int i = tid; i < n; i += SMP_THREADS) m = fmaxf(m, __fdiv_rn(smp_clean(logits[i]), tc));
    m = smp_block_max(S, m);
    float s = 0.f;
    for (int i = tid; i < n; i += SMP_THREADS) s += expf(__fsub_rn(__fdiv_rn(smp_clean(logits[i]), tc), m));
    s = smp_block_sum(S, s);
    if (!(s > 0.f)) {
      pick = smp_first_max(S, n, lkey, all);
    } else {
      for (int i = tid; i < n; i += SMP_THREADS) p[i] = __fdiv_rn(expf(__fsub_rn(__fdiv_rn(smp_clean(logits[i]), tc), m)), s);
      __syncthreads();
      auto pkey = [&](int i) { return __float_as_uint(p[i]); };
      auto pmass = [&](int i) { return smp_fix(p[i]); };
      // the nucleus: entries above the crossing of top_p, and the crossing one; the top entry alone
      // when the running sum never exceeds top_p
      int c = smp_select(S, n, smp_fix(top_p), pkey, pmass, all);
      if (c < 0) c = smp_first_max(S, n, pkey, all);
      const uint32_t kc = __float_as_uint(p[c]);
      auto in_nucleus = [&](int i) {
        const uint32_t k = __float_as_uint(p[i]);
        return k > kc || (k == kc && i <= c);
      };
      unsigned long long ps = 0ull;
      for (int i = tid; i < n; i += SMP_THREADS)
        if (in_nucleus(i)) ps += smp_fix(p[i]);
      ps = smp_block_sum_u64(S, ps);
      const float P = (float)((double)ps / SMP_ONE);
      const int top = smp_first_max(S, n, pkey, all);
      if (!(P > 0.f)) {
        pick = top;
      } else {
        // choice: the entry where the running sum of p / P crosses u times its total
        auto nmass = [&](int i) { return smp_fix(__fdiv_rn(p[i], P)); };
        unsigned long long tot = 0ull;
        for (int i = tid; i < n; i += SMP_THREADS)
          if (in_nucleus(i)) tot += nmass(i);
        tot = smp_block_sum_u64(S, tot);
        const double uu = u_index ? u[*u_index] : u[0];
        const unsigned long long target = (unsigned long long)(uu * (double)tot);
        pick = smp_select(S, n, target, pkey, nmass, in_nucleus);
        if (pick < 0) {  // u * total rounded to the total: the last entry of the nucleus
          pick = c;
        }
      }
    }
  }
  if (tid == 0) {
    if (index_out) *index_out = pick;
    // the greedy-argmax key format, so that gsdlq_greedy_advance takes the pick
    if (key_out) *key_out = (1ull << 32) | (unsigned long long)(0xffffffffu - (uint32_t)pick);
  }
}

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_sample_work_size(int n, size_t* bytes) {
  if (!bytes || n <= 0) return GSDLQ_ERR_INVALID;
  *bytes = sizeof(float) * (size_t)n;
  return GSDLQ_OK;
}

extern "C" int gsdlq_sample_top_p(const float* logits, int n, float temperature, float top_p, const double* u,
                                  const int* u_index, void* work, size_t work_bytes, unsigned long long* argmax_key,
                                  int* out_index, gsdlq_stream_t stream) {
  if (!logits || n <= 0 || !u || !work || work_bytes < sizeof(float) * (size_t)n) return GSDLQ_ERR_INVALID;
  if (!argmax_key && !out_index) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(work) & 3u) return GSDLQ_ERR_INVALID;
  sample_kernel<<<1, SMP_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, n, temperature, top_p, u, u_index, static_cast<float*>(work), argmax_key, out_index);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

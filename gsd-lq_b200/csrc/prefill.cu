// prefill.cu -- the row-batched kernels of chunked prefill: a chunk of n prompt tokens goes through each
// packed linear as one tensor-core dequant-GEMM (gsdlq_hex2d_matmul), and through these kernels around
// it.  Each is the reference's per-token operation applied to every row of the chunk:
//
//   gsdlq_embed_rows      x[t] = f32(embed[ids[t]])                    (gsd_lq_cpu_runtime.py:303)
//   gsdlq_rmsnorm_rows    out[t] = x[t] * (1/sqrt(mean(x[t]^2) + eps)) * w  (gsd_lq_cpu_engine.c:67-82)
//   gsdlq_rope_kv_rows    RoPE of q[t], k[t] at position pos0 + t, fp16 K/V into the cache
//                         (gsd_lq_cpu_engine.c:186-262; angles from the host table of gsdlq_rope_table)
//   gsdlq_attention_rows  causal GQA attention of token t over positions 0 .. pos0 + t
//                         (gsd_lq_cpu_engine.c:265-330 per token)
//
// The reference has no batched prefill: it runs forward_token once per prompt token
// (run_gpu_native_chat.py:1128-1131).
#include <cmath>

#include "common.cuh"

namespace gsdlq {

__global__ void embed_rows_kernel(const uint16_t* __restrict__ embed, const int* __restrict__ ids, int vocab, int dim,
                                  float* __restrict__ out) {
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) raise_flag(GSDLQ_FLAG_BAD_TOKEN);
    id = 0;
  }
  const uint16_t* row = embed + (size_t)id * dim;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) out[(size_t)t * dim + c] = h2f(row[c]);
}

__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
                                    int dim, float eps) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += xr[i] * xr[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(t / (float)dim + eps);
  }
  __syncthreads();
  const float inv = red[0];
  float* o = out + (size_t)blockIdx.x * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// one CTA per token: interleaved pairs (2i, 2i+1) of every q and k head rotated by (cos, sin) of the
// token's position; k (rotated) and v stored as fp16 at [layer][pos][kv head][dim]
__global__ void rope_kv_rows_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                    uint16_t* __restrict__ kc, uint16_t* __restrict__ vc,
                                    const float2* __restrict__ cs, int layer, int pos0, int n_heads, int n_kv, int hd,
                                    int max_seq) {
  const int t = blockIdx.x, pos = pos0 + t, half = hd / 2;
  if (pos < 0 || pos >= max_seq) {
    if (threadIdx.x == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
    return;
  }
  const float2* c = cs + (size_t)pos * half;
  float* qt = q + (size_t)t * n_heads * hd;
  for (int e = threadIdx.x; e < n_heads * half; e += blockDim.x) {
    const int h = e / half, i = e - h * half;
    float* p = qt + (size_t)h * hd + 2 * i;
    const float a = p[0], b = p[1];
    const float2 r = c[i];
    p[0] = __fsub_rn(__fmul_rn(a, r.x), __fmul_rn(b, r.y));
    p[1] = __fadd_rn(__fmul_rn(a, r.y), __fmul_rn(b, r.x));
  }
  const size_t base = ((size_t)layer * max_seq + pos) * n_kv * hd;
  const float* kt = k + (size_t)t * n_kv * hd;
  const float* vt = v + (size_t)t * n_kv * hd;
  for (int e = threadIdx.x; e < n_kv * half; e += blockDim.x) {
    const int h = e / half, i = e - h * half;
    const size_t o = (size_t)h * hd + 2 * i;
    const float a = kt[o], b = kt[o + 1];
    const float2 r = c[i];
    kc[base + o] = f2h(__fsub_rn(__fmul_rn(a, r.x), __fmul_rn(b, r.y)));
    kc[base + o + 1] = f2h(__fadd_rn(__fmul_rn(a, r.y), __fmul_rn(b, r.x)));
    vc[base + o] = f2h(vt[o]);
    vc[base + o + 1] = f2h(vt[o + 1]);
  }
}

// Causal attention of one token's GQA group: CTA (token t, kv head g), 128 threads.  Positions go in
// tiles of 32: thread (position j, head h) computes the score q_h . k_j * sm_scale, each head's running
// maximum and sum are updated (online softmax), and thread d accumulates every head's sum of p_j v_j[d].
constexpr int AR_THREADS = 128, AR_TILE = 32, AR_MAXGQ = 8, AR_MAXHD = 128;
__global__ void __launch_bounds__(AR_THREADS) attention_rows_kernel(const float* __restrict__ q,
                                                                    const uint16_t* __restrict__ kc,
                                                                    const uint16_t* __restrict__ vc,
                                                                    float* __restrict__ out, int layer, int pos0,
                                                                    int n_heads, int n_kv, int hd, int max_seq,
                                                                    float sm_scale) {
  __shared__ float qs[AR_MAXGQ][AR_MAXHD];
  __shared__ float ps[AR_MAXGQ][AR_TILE];
  __shared__ float s_m[AR_MAXGQ], s_l[AR_MAXGQ], s_f[AR_MAXGQ];
  const int t = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
  const int gq = n_heads / n_kv, pos = pos0 + t;
  const int len = (pos >= 0 && pos < max_seq) ? pos + 1 : 0;
  if (len == 0 && tid == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
  const float* qt = q + ((size_t)t * n_heads + (size_t)g * gq) * hd;
  for (int e = tid; e < gq * hd; e += AR_THREADS) qs[e / hd][e % hd] = qt[e];
  if (tid < gq) {
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.f;
  }
  float acc[AR_MAXGQ];
#pragma unroll
  for (int h = 0; h < AR_MAXGQ; ++h) acc[h] = 0.f;
  __syncthreads();
  const size_t stride = (size_t)n_kv * hd;
  const uint16_t* kl = kc + (size_t)layer * max_seq * stride + (size_t)g * hd;
  const uint16_t* vl = vc + (size_t)layer * max_seq * stride + (size_t)g * hd;
  for (int j0 = 0; j0 < len; j0 += AR_TILE) {
    // scores of the tile: thread (j, h) for j = tid % 32, heads h = tid / 32, + 4, ...
    for (int e = tid; e < gq * AR_TILE; e += AR_THREADS) {
      const int h = e / AR_TILE, j = e - h * AR_TILE, p = j0 + j;
      float s = -INFINITY;
      if (p < len) {
        const uint16_t* kr = kl + (size_t)p * stride;
        float d = 0.f;
        for (int i = 0; i < hd; i += 2) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(kr + i);
          d = fmaf(qs[h][i], h2f((uint16_t)(w & 0xffffu)), d);
          d = fmaf(qs[h][i + 1], h2f((uint16_t)(w >> 16)), d);
        }
        s = d * sm_scale;
      }
      ps[h][j] = s;
    }
    __syncthreads();
    // online softmax: one warp per head
    const int warp = tid >> 5, lane = tid & 31;
    for (int h = warp; h < gq; h += AR_THREADS / 32) {
      const float s = ps[h][lane];
      const float mt = warp_max(s);
      const float m_old = s_m[h], m_new = fmaxf(m_old, mt);
      const float p = (s == -INFINITY) ? 0.f : expf(s - m_new);
      const float sum = warp_sum(p);
      ps[h][lane] = p;
      __syncwarp();
      if (lane == 0) {
        const float f = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        s_f[h] = f;
        s_l[h] = s_l[h] * f + sum;
        s_m[h] = m_new;
      }
    }
    __syncthreads();
    // P.V: thread d (< hd) for every head
    if (tid < hd) {
      float vcol[AR_TILE];
#pragma unroll
      for (int j = 0; j < AR_TILE; ++j) vcol[j] = (j0 + j < len) ? h2f(vl[(size_t)(j0 + j) * stride + tid]) : 0.f;
      for (int h = 0; h < gq; ++h) {
        float a = acc[h] * s_f[h];
#pragma unroll
        for (int j = 0; j < AR_TILE; ++j) a = fmaf(ps[h][j], vcol[j], a);
        acc[h] = a;
      }
    }
    __syncthreads();
  }
  if (tid < hd) {
    float* ot = out + ((size_t)t * n_heads + (size_t)g * gq) * hd;
    for (int h = 0; h < gq; ++h) ot[(size_t)h * hd + tid] = len > 0 ? acc[h] / s_l[h] : 0.f;
  }
}

}  // namespace gsdlq

using namespace gsdlq;

extern "C" {

int gsdlq_embed_rows(const uint16_t* embed, const int* ids, int n, int vocab, int dim, float* out, gsdlq_stream_t stream) {
  if (!embed || !ids || !out || n <= 0 || vocab <= 0 || dim <= 0) return GSDLQ_ERR_INVALID;
  embed_rows_kernel<<<n, 256, 0, static_cast<cudaStream_t>(stream)>>>(embed, ids, vocab, dim, out);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_rmsnorm_rows(const float* x, const float* w, float* out, int n, int dim, float eps, gsdlq_stream_t stream) {
  if (!x || !w || !out || n <= 0 || dim <= 0) return GSDLQ_ERR_INVALID;
  rmsnorm_rows_kernel<<<n, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, w, out, dim, eps);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_rope_kv_rows(float* q, const float* k, const float* v, uint16_t* k_cache, uint16_t* v_cache,
                       const float* rope_cs, int layer, int pos0, int n, int n_heads, int n_kv_heads, int head_dim,
                       int max_seq, gsdlq_stream_t stream) {
  if (!q || !k || !v || !k_cache || !v_cache || !rope_cs || n <= 0 || layer < 0 || pos0 < 0 || max_seq <= 0)
    return GSDLQ_ERR_INVALID;
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2) return GSDLQ_ERR_INVALID;
  if (pos0 + n > max_seq) return GSDLQ_ERR_INVALID;
  rope_kv_rows_kernel<<<n, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, k_cache, v_cache, reinterpret_cast<const float2*>(rope_cs), layer, pos0, n_heads, n_kv_heads, head_dim,
      max_seq);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_attention_rows(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, float* out, int layer,
                         int pos0, int n, int n_heads, int n_kv_heads, int head_dim, int max_seq, float sm_scale,
                         gsdlq_stream_t stream) {
  if (!q || !k_cache || !v_cache || !out || n <= 0 || layer < 0 || pos0 < 0 || pos0 + n > max_seq) return GSDLQ_ERR_INVALID;
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > AR_MAXGQ) return GSDLQ_ERR_INVALID;
  if (head_dim <= 0 || head_dim > AR_MAXHD || head_dim % 2) return GSDLQ_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 3u) return GSDLQ_ERR_INVALID;
  attention_rows_kernel<<<dim3(n, n_kv_heads), AR_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k_cache, v_cache, out, layer, pos0, n_heads, n_kv_heads, head_dim, max_seq, sm_scale);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

}  // extern "C"

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
#include <atomic>
#include <algorithm>
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
// With pos_dev (batched decode): row t is sequence t, at position pos_dev[t], with its own cache at
// seq_stride elements after the previous sequence's.
__global__ void rope_kv_rows_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                    uint16_t* __restrict__ kc, uint16_t* __restrict__ vc,
                                    const float2* __restrict__ cs, int layer, int pos0, int n_heads, int n_kv, int hd,
                                    int max_seq, const int* __restrict__ pos_dev, size_t seq_stride,
                                    int row_stride) {
  const int t = blockIdx.x, pos = pos_dev ? pos_dev[t] : pos0 + t, half = hd / 2;
  // row t of q, k, v: row_stride elements apart (0: packed, [n][heads][hd])
  if (pos_dev) {
    kc += (size_t)t * seq_stride;
    vc += (size_t)t * seq_stride;
  }
  if (pos < 0 || pos >= max_seq) {
    if (threadIdx.x == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
    return;
  }
  const float2* c = cs + (size_t)pos * half;
  float* qt = q + (size_t)t * (row_stride ? row_stride : n_heads * hd);
  for (int e = threadIdx.x; e < n_heads * half; e += blockDim.x) {
    const int h = e / half, i = e - h * half;
    float* p = qt + (size_t)h * hd + 2 * i;
    const float a = p[0], b = p[1];
    const float2 r = c[i];
    p[0] = __fsub_rn(__fmul_rn(a, r.x), __fmul_rn(b, r.y));
    p[1] = __fadd_rn(__fmul_rn(a, r.y), __fmul_rn(b, r.x));
  }
  const size_t base = ((size_t)layer * max_seq + pos) * n_kv * hd;
  const float* kt = k + (size_t)t * (row_stride ? row_stride : n_kv * hd);
  const float* vt = v + (size_t)t * (row_stride ? row_stride : n_kv * hd);
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

// Causal attention of a chunk, tiled: CTA (block of AT_ROWS query rows, kv head g, split z).  The rows
// are (token, head) pairs of one GQA group, token-major: row r is token t0 + r / gq, head g * gq + r % gq,
// so every row of the CTA reads the same K and V.  Positions go in tiles of AT_POS: the fp16 K tile is
// converted into shared memory transposed (kT[d][j]), V as is (vs[j][d]); thread (rg = tid / 16,
// pg = tid % 16) computes the scores of rows 4rg .. 4rg+3 at positions 4pg .. 4pg+3 from float4 reads of
// the pre-scaled qT[d][r] and of kT, runs the online softmax of its rows in registers (the 16 threads of a
// row group are one half-warp, reduced by shuffles), writes its p into pT[j][r] and accumulates
// out[4 rows][4 dims per 64] += p v.  With splits > 1 each split covers a contiguous range of the CTA's
// position tiles and writes its unnormalised rows with their (max, sum) into the work buffer, and
// attention_combine_kernel merges the splits.
constexpr int AT_THREADS = 128, AT_ROWS = 32, AT_POS = 64, AT_MAXGQ = 8, AT_MAXSPLIT = 8;

__host__ __device__ constexpr size_t at_smem_bytes(int hd) {
  return sizeof(float) * ((size_t)hd * AT_ROWS + (size_t)hd * AT_POS + (size_t)AT_POS * hd + (size_t)AT_POS * AT_ROWS);
}

// swizzled float4 slot of row group rg in pT row j (spreads the row groups' stores over the banks)
__device__ __forceinline__ int pt_slot(int j, int rg) { return j * AT_ROWS + 4 * (rg ^ ((j >> 2) & 7)); }

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, 2)
    attention_rows_kernel(const float* __restrict__ q, const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc,
                          float* __restrict__ out, float* __restrict__ work, int layer, int pos0, int n, int n_heads,
                          int n_kv, int max_seq, float sm_scale, int splits) {
  constexpr int DC = HD / 64;  // 64-dim column groups of the thread's output
  extern __shared__ __align__(16) float at_smem[];
  float* qT = at_smem;                  // [HD][AT_ROWS]
  float* kT = qT + HD * AT_ROWS;        // [HD][AT_POS]
  float* vs = kT + HD * AT_POS;         // [AT_POS][HD]
  float* pT = vs + AT_POS * HD;         // [AT_POS][AT_ROWS], swizzled slots
  const int tid = threadIdx.x, rg = tid >> 4, pg = tid & 15;
  const int g = blockIdx.y, z = blockIdx.z;
  const int gq = n_heads / n_kv, qb = AT_ROWS / gq, used = qb * gq;
  const int t0 = blockIdx.x * qb;
  const int t_last = min(t0 + qb, n) - 1;
  // rows past the chunk (or past qb * gq) repeat the last valid row and are not written
  int lim[4], tok[4], head[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = rg * 4 + i;
    int t = r < used ? t0 + r / gq : t_last;
    t = min(t, t_last);
    tok[i] = (r < used && t0 + r / gq <= t_last) ? t : -1;
    head[i] = g * gq + (r < used ? r % gq : 0);
    lim[i] = pos0 + t;
  }
  // q rows, pre-scaled, transposed
  for (int e = tid; e < AT_ROWS * HD; e += AT_THREADS) {
    const int r = e / HD, d = e - r * HD;
    int t = r < used ? t0 + r / gq : t_last;
    t = min(t, t_last);
    const int h = g * gq + (r < used ? r % gq : 0);
    qT[d * AT_ROWS + r] = q[((size_t)t * n_heads + h) * HD + d] * sm_scale;
  }
  const int ntiles = (pos0 + t_last) / AT_POS + 1;
  const int per = (ntiles + splits - 1) / splits;
  const int tile0 = z * per, tile1 = min(ntiles, tile0 + per);
  const size_t stride = (size_t)n_kv * HD;
  const uint16_t* kl = kc + (size_t)layer * max_seq * stride + (size_t)g * HD;
  const uint16_t* vl = vc + (size_t)layer * max_seq * stride + (size_t)g * HD;
  const int kv_end = pos0 + t_last + 1;  // positions written so far for the CTA's last token
  float m[4], lsum[4], acc[4][4 * DC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    lsum[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4 * DC; ++c) acc[i][c] = 0.f;
  }
  for (int tile = tile0; tile < tile1; ++tile) {
    const int j0 = tile * AT_POS;
    __syncthreads();  // the previous tile's kT / vs / pT are consumed (and qT written, on the first tile)
    // K: lanes walk positions (conflict-free transposed stores); V: lanes walk dims (coalesced rows)
#pragma unroll 4
    for (int e = tid; e < AT_POS * HD / 8; e += AT_THREADS) {
      const int j = e % AT_POS, d8 = e / AT_POS, p = j0 + j;
      uint4 w = make_uint4(0, 0, 0, 0);
      if (p < kv_end) w = __ldg(reinterpret_cast<const uint4*>(kl + (size_t)p * stride + d8 * 8));
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kT[(d8 * 8 + 2 * i) * AT_POS + j] = h2f((uint16_t)(ww[i] & 0xffffu));
        kT[(d8 * 8 + 2 * i + 1) * AT_POS + j] = h2f((uint16_t)(ww[i] >> 16));
      }
    }
#pragma unroll 4
    for (int e = tid; e < AT_POS * HD / 8; e += AT_THREADS) {
      const int d8 = e % (HD / 8), j = e / (HD / 8), p = j0 + j;
      uint4 w = make_uint4(0, 0, 0, 0);
      if (p < kv_end) w = __ldg(reinterpret_cast<const uint4*>(vl + (size_t)p * stride + d8 * 8));
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
      float4* dst = reinterpret_cast<float4*>(vs + j * HD + d8 * 8);
      dst[0] = make_float4(h2f((uint16_t)(ww[0] & 0xffffu)), h2f((uint16_t)(ww[0] >> 16)),
                           h2f((uint16_t)(ww[1] & 0xffffu)), h2f((uint16_t)(ww[1] >> 16)));
      dst[1] = make_float4(h2f((uint16_t)(ww[2] & 0xffffu)), h2f((uint16_t)(ww[2] >> 16)),
                           h2f((uint16_t)(ww[3] & 0xffffu)), h2f((uint16_t)(ww[3] >> 16)));
    }
    __syncthreads();
    // scores of rows 4rg.. at positions 4pg..
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
#pragma unroll 8
    for (int d = 0; d < HD; ++d) {
      const float4 qv = *reinterpret_cast<const float4*>(qT + d * AT_ROWS + rg * 4);
      const float4 kv = *reinterpret_cast<const float4*>(kT + d * AT_POS + pg * 4);
      const float qq[4] = {qv.x, qv.y, qv.z, qv.w}, kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[i][c] = fmaf(qq[i], kk[c], s[i][c]);
    }
    // online softmax per row, reduced over the half-warp of the row group
    float f[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (j0 + pg * 4 + c > lim[i]) s[i][c] = -INFINITY;
        tmax = fmaxf(tmax, s[i][c]);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mn = fmaxf(m[i], tmax);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[i][c] = (s[i][c] == -INFINITY) ? 0.f : expf(s[i][c] - mn);
        rs += s[i][c];
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
      f[i] = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
      if (mn == -INFINITY) f[i] = 1.f;
      lsum[i] = lsum[i] * f[i] + rs;
      m[i] = mn;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<float4*>(pT + pt_slot(pg * 4 + c, rg)) = make_float4(s[0][c], s[1][c], s[2][c], s[3][c]);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4 * DC; ++c) acc[i][c] *= f[i];
    __syncthreads();
    // out rows 4rg.. at dims 4pg + 64 c ..
#pragma unroll 4
    for (int j = 0; j < AT_POS; ++j) {
      const float4 pv = *reinterpret_cast<const float4*>(pT + pt_slot(j, rg));
      const float pp[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int dc = 0; dc < DC; ++dc) {
        const float4 vv = *reinterpret_cast<const float4*>(vs + j * HD + dc * 64 + pg * 4);
        const float v4[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[i][dc * 4 + c] = fmaf(pp[i], v4[c], acc[i][dc * 4 + c]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (tok[i] < 0) continue;
    const size_t row = (size_t)tok[i] * n_heads + head[i];
    if (splits == 1) {
      const float inv = 1.0f / lsum[i];
#pragma unroll
      for (int dc = 0; dc < DC; ++dc)
        *reinterpret_cast<float4*>(out + row * HD + dc * 64 + pg * 4) =
            make_float4(acc[i][dc * 4] * inv, acc[i][dc * 4 + 1] * inv, acc[i][dc * 4 + 2] * inv, acc[i][dc * 4 + 3] * inv);
    } else {
      const size_t rows = (size_t)n * n_heads;
      float* wa = work + ((size_t)z * rows + row) * HD;
#pragma unroll
      for (int dc = 0; dc < DC; ++dc)
        *reinterpret_cast<float4*>(wa + dc * 64 + pg * 4) =
            make_float4(acc[i][dc * 4], acc[i][dc * 4 + 1], acc[i][dc * 4 + 2], acc[i][dc * 4 + 3]);
      if (pg == 0) {
        float* wm = work + (size_t)AT_MAXSPLIT * rows * HD;
        wm[((size_t)z * rows + row) * 2] = m[i];
        wm[((size_t)z * rows + row) * 2 + 1] = lsum[i];
      }
    }
  }
}

// merge of the splits of row (token blockIdx.x, head blockIdx.y): out = sum_z e^(m_z - M) acc_z / L
__global__ void attention_combine_kernel(const float* __restrict__ work, float* __restrict__ out, int n, int n_heads,
                                         int hd, int splits) {
  const size_t rows = (size_t)n * n_heads, row = (size_t)blockIdx.x * n_heads + blockIdx.y;
  const float* wm = work + (size_t)AT_MAXSPLIT * rows * hd;
  float mx = -INFINITY;
  for (int z = 0; z < splits; ++z) mx = fmaxf(mx, wm[((size_t)z * rows + row) * 2]);
  float l = 0.f, a = 0.f;
  for (int z = 0; z < splits; ++z) {
    const float mz = wm[((size_t)z * rows + row) * 2];
    if (mz == -INFINITY) continue;
    const float e = expf(mz - mx);
    l = fmaf(wm[((size_t)z * rows + row) * 2 + 1], e, l);
    a = fmaf(work[((size_t)z * rows + row) * hd + threadIdx.x], e, a);
  }
  out[row * hd + threadIdx.x] = a / l;
}

// Batched decode attention: sequence b's one query token (at position pos[b], its K/V already appended)
// over positions 0 .. pos[b] of its own cache.  CTA (sequence b, kv head g, split z), 4 warps; the split
// covers a contiguous range of 32-position tiles, dealt to the warps in turn.  Lane j of a warp scores
// position 32 tile + j against the GQ query heads (its K row read whole, q from shared memory), the
// warp keeps each head's running max and sum (online softmax), and the P.V step runs lanes over head
// dimensions (HD / 32 each) with each position's weight broadcast, reading V rows whole.  The warps'
// partials merge in shared memory; with splits > 1 the CTA writes its unnormalised rows and (max, sum)
// for attention_combine_kernel, as gsdlq_attention_rows does.
constexpr int AD_THREADS = 128;
template <int HD, int GQ>
__global__ void __launch_bounds__(AD_THREADS)
    attention_decode_kernel(const float* __restrict__ q, const uint16_t* __restrict__ kc,
                            const uint16_t* __restrict__ vc, size_t seq_stride, float* __restrict__ out,
                            float* __restrict__ work, int layer, const int* __restrict__ pos, int B, int n_heads,
                            int n_kv, int max_seq, float sm_scale, int splits, int q_stride) {
  constexpr int DL = HD / 32;  // dimensions per lane in the P.V step
  __shared__ float qs[GQ][HD];
  __shared__ float wm[4][GQ], wl[4][GQ];
  __shared__ float wacc[4][GQ][HD];
  const int b = blockIdx.x, g = blockIdx.y, z = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int p_last = pos[b];
  const bool ok = p_last >= 0 && p_last < max_seq;
  if (!ok && tid == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
  const int len = ok ? p_last + 1 : 0;
  const float* qb = q + (size_t)b * (q_stride ? q_stride : n_heads * HD) + (size_t)g * GQ * HD;
  for (int e = tid; e < GQ * HD; e += AD_THREADS) qs[e / HD][e % HD] = qb[e] * sm_scale;
  __syncthreads();
  const size_t stride = (size_t)n_kv * HD;
  const uint16_t* kl = kc + (size_t)b * seq_stride + (size_t)layer * max_seq * stride + (size_t)g * HD;
  const uint16_t* vl = vc + (size_t)b * seq_stride + (size_t)layer * max_seq * stride + (size_t)g * HD;
  const int ntiles = (len + 31) / 32, per = (ntiles + splits - 1) / splits;
  const int tile0 = z * per, tile1 = min(ntiles, tile0 + per);
  float m[GQ], l[GQ], acc[GQ][DL];
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) acc[h][d] = 0.f;
  }
  for (int tile = tile0 + warp; tile < tile1; tile += 4) {
    const int p = tile * 32 + lane;
    float s[GQ];
#pragma unroll
    for (int h = 0; h < GQ; ++h) s[h] = 0.f;
    if (p < len) {
      const uint4* kr = reinterpret_cast<const uint4*>(kl + (size_t)p * stride);
      uint4 kv[HD / 8];
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) kv[c] = __ldg(kr + c);
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) {
        const uint32_t w4[4] = {kv[c].x, kv[c].y, kv[c].z, kv[c].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float k0 = h2f((uint16_t)(w4[t] & 0xffffu)), k1 = h2f((uint16_t)(w4[t] >> 16));
#pragma unroll
          for (int h = 0; h < GQ; ++h) s[h] = fmaf(qs[h][8 * c + 2 * t + 1], k1, fmaf(qs[h][8 * c + 2 * t], k0, s[h]));
        }
      }
    }
    float pw[GQ];
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
      const float sv = p < len ? s[h] : -INFINITY;
      const float mt = warp_max(sv);
      const float mn = fmaxf(m[h], mt);  // finite: the tile holds at least one position
      pw[h] = p < len ? expf(sv - mn) : 0.f;
      const float f = m[h] == -INFINITY ? 0.f : expf(m[h] - mn);
      l[h] = l[h] * f + warp_sum(pw[h]);
      m[h] = mn;
#pragma unroll
      for (int d = 0; d < DL; ++d) acc[h][d] *= f;
    }
    // P.V: eight positions' V rows loaded together, then their weights broadcast and applied
    const int nvalid = min(32, len - tile * 32);
    for (int j0 = 0; j0 < nvalid; j0 += 8) {
      float vv[8][DL];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int j = min(j0 + jj, nvalid - 1);  // past the tile's last position: re-read it, weight 0 below
        const uint16_t* vr = vl + (size_t)(tile * 32 + j) * stride + lane * DL;
        if (DL == 4) {
          const uint2 w2 = __ldg(reinterpret_cast<const uint2*>(vr));
          vv[jj][0] = h2f((uint16_t)(w2.x & 0xffffu));
          vv[jj][1 % DL] = h2f((uint16_t)(w2.x >> 16));
          vv[jj][2 % DL] = h2f((uint16_t)(w2.y & 0xffffu));
          vv[jj][3 % DL] = h2f((uint16_t)(w2.y >> 16));
        } else {
          const uint32_t w1 = __ldg(reinterpret_cast<const uint32_t*>(vr));
          vv[jj][0] = h2f((uint16_t)(w1 & 0xffffu));
          vv[jj][1 % DL] = h2f((uint16_t)(w1 >> 16));
        }
      }
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
          float pj = __shfl_sync(0xffffffffu, pw[h], (j0 + jj) & 31);
          if (j0 + jj >= nvalid) pj = 0.f;
#pragma unroll
          for (int d = 0; d < DL; ++d) acc[h][d] = fmaf(pj, vv[jj][d], acc[h][d]);
        }
      }
    }
  }
  // merge the warps
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
      wm[warp][h] = m[h];
      wl[warp][h] = l[h];
    }
  }
#pragma unroll
  for (int h = 0; h < GQ; ++h)
#pragma unroll
    for (int d = 0; d < DL; ++d) wacc[warp][h][lane * DL + d] = acc[h][d];
  __syncthreads();
  const size_t rows = (size_t)B * n_heads;
  for (int e = tid; e < GQ * HD; e += AD_THREADS) {
    const int h = e / HD, d = e % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][h]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (wm[w][h] == -INFINITY) continue;
      const float f = expf(wm[w][h] - M);
      L = fmaf(wl[w][h], f, L);
      A = fmaf(wacc[w][h][d], f, A);
    }
    const size_t row = (size_t)b * n_heads + (size_t)g * GQ + h;
    if (splits == 1) {
      out[row * HD + d] = L > 0.f ? A / L : 0.f;
    } else {
      work[((size_t)z * rows + row) * HD + d] = A;
      if (d == 0) {
        float* wmw = work + (size_t)AT_MAXSPLIT * rows * HD;
        wmw[((size_t)z * rows + row) * 2] = M;
        wmw[((size_t)z * rows + row) * 2 + 1] = L;
      }
    }
  }
}

// Greedy pick per row of a batch of logits (the reference's greedy sample_token: NaN -> -1e4, +inf -> 100,
// -inf -> -1e4, the first maximum) and the batch's bookkeeping: ids[b] = pick; out_ids[b][pos[b] + 1] =
// pick (when out_ids); pos[b] += 1 (when pos).
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ logits, int n, int* __restrict__ ids,
                                                          int* __restrict__ pos, int* __restrict__ out_ids,
                                                          int out_stride) {
  __shared__ unsigned long long red[32];
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* lr = logits + (size_t)b * n;
  unsigned long long best = 0ull;
  for (int i = tid; i < n; i += 1024) {
    float v = lr[i];
    v = isnan(v) ? -1e4f : (isinf(v) ? (v > 0.f ? 100.f : -1e4f) : v) + 0.0f;
    const uint32_t bits = __float_as_uint(v);
    const uint32_t key = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    const unsigned long long k = ((unsigned long long)key << 32) | (0xffffffffu - (uint32_t)i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(0xffffffffu, best, o);
    best = u > best ? u : best;
  }
  if ((tid & 31) == 0) red[tid >> 5] = best;
  __syncthreads();
  if (tid < 32) {
    best = red[tid];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long u = __shfl_xor_sync(0xffffffffu, best, o);
      best = u > best ? u : best;
    }
    if (tid == 0) {
      const int pick = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffull));
      ids[b] = pick;
      if (pos) {
        const int p = pos[b];
        if (out_ids && p + 1 >= 0 && p + 1 < out_stride) out_ids[(size_t)b * out_stride + p + 1] = pick;
        pos[b] = p + 1;
      }
    }
  }
}

// gsd_cpu_swiglu (gsd_lq_cpu_engine.c:97-108) of rows laid out [gate | up]: out[r][i] = silu(g) * u with
// g = gate_up[r][i], u = gate_up[r][n + i] (the output of one linear over the stacked gate and up rows)
__global__ void swiglu_rows_kernel(const float* __restrict__ gu, float* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
  if (i < n) {
    const float g = gu[(size_t)r * 2 * n + i];
    out[(size_t)r * n + i] = (g / (1.0f + expf(-g))) * gu[(size_t)r * 2 * n + n + i];
  }
}

static size_t attention_rows_work(int n, int n_heads, int hd) {
  return sizeof(float) * (size_t)AT_MAXSPLIT * n * n_heads * (hd + 2);
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
      max_seq, nullptr, 0, 0);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_rope_kv_batch(float* q, const float* k, const float* v, int row_stride, uint16_t* k_cache,
                        uint16_t* v_cache, size_t seq_stride, const float* rope_cs, int layer, const int* pos, int batch,
                        int n_heads, int n_kv_heads, int head_dim, int max_seq, gsdlq_stream_t stream) {
  if (!q || !k || !v || !k_cache || !v_cache || !rope_cs || !pos || batch <= 0 || layer < 0 || max_seq <= 0)
    return GSDLQ_ERR_INVALID;
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2) return GSDLQ_ERR_INVALID;
  if (seq_stride < (size_t)(layer + 1) * max_seq * n_kv_heads * head_dim) return GSDLQ_ERR_INVALID;
  if (row_stride < 0 || (row_stride > 0 && row_stride < n_heads * head_dim)) return GSDLQ_ERR_INVALID;
  rope_kv_rows_kernel<<<batch, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, k_cache, v_cache, reinterpret_cast<const float2*>(rope_cs), layer, 0, n_heads, n_kv_heads, head_dim,
      max_seq, pos, seq_stride, row_stride);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_attention_rows_work_size(int n, int n_heads, int head_dim, size_t* bytes) {
  if (!bytes || n <= 0 || n_heads <= 0 || head_dim <= 0) return GSDLQ_ERR_INVALID;
  *bytes = attention_rows_work(n, n_heads, head_dim);
  return GSDLQ_OK;
}

int gsdlq_attention_rows(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, float* out, void* work,
                         size_t work_bytes, int layer, int pos0, int n, int n_heads, int n_kv_heads, int head_dim,
                         int max_seq, float sm_scale, gsdlq_stream_t stream) {
  if (!q || !k_cache || !v_cache || !out || !work || n <= 0 || layer < 0 || pos0 < 0 || pos0 + n > max_seq)
    return GSDLQ_ERR_INVALID;
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > AT_MAXGQ) return GSDLQ_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return GSDLQ_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(work)) & 15u)
    return GSDLQ_ERR_INVALID;
  if (work_bytes < attention_rows_work(n, n_heads, head_dim)) return GSDLQ_ERR_INVALID;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int gq = n_heads / n_kv_heads, qb = AT_ROWS / gq;
  const int blocks = (n + qb - 1) / qb;
  // splits of the position range so that about two CTAs per SM are busy; none shorter than one tile
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int base = blocks * n_kv_heads, tiles = (pos0 + n - 1) / AT_POS + 1;
  int splits = (2 * sms + base - 1) / base;
  splits = std::max(1, std::min(std::min(splits, AT_MAXSPLIT), tiles));
  const dim3 grid(blocks, n_kv_heads, splits);
  float* wk = static_cast<float*>(work);
  // the 88 KB of the head_dim-128 tiles need the opt-in size, set once per device
  static std::atomic<bool> smem_set[64];
  const int di = (dev >= 0 && dev < 64) ? dev : 0;
  if (!smem_set[di].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(attention_rows_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)at_smem_bytes(128));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_rows_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)at_smem_bytes(64));
    if (e != cudaSuccess) return record_cuda_error(e);
    smem_set[di].store(true, std::memory_order_release);
  }
  if (head_dim == 128) {
    attention_rows_kernel<128><<<grid, AT_THREADS, at_smem_bytes(128), st>>>(
        q, k_cache, v_cache, out, wk, layer, pos0, n, n_heads, n_kv_heads, max_seq, sm_scale, splits);
  } else {
    attention_rows_kernel<64><<<grid, AT_THREADS, at_smem_bytes(64), st>>>(
        q, k_cache, v_cache, out, wk, layer, pos0, n, n_heads, n_kv_heads, max_seq, sm_scale, splits);
  }
  GSDLQ_CUDA_CHECK_LAUNCH();
  if (splits > 1) {
    attention_combine_kernel<<<dim3(n, n_heads), head_dim, 0, st>>>(wk, out, n, n_heads, head_dim, splits);
    GSDLQ_CUDA_CHECK_LAUNCH();
  }
  return GSDLQ_OK;
}

int gsdlq_swiglu_rows(const float* gate_up, float* out, int rows, int n, gsdlq_stream_t stream) {
  if (!gate_up || !out || rows <= 0 || n <= 0) return GSDLQ_ERR_INVALID;
  swiglu_rows_kernel<<<dim3((n + 255) / 256, rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(gate_up, out, n);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_argmax_rows(const float* logits, int rows, int n, int* ids, int* pos, int* out_ids, int out_stride,
                      gsdlq_stream_t stream) {
  if (!logits || !ids || rows <= 0 || n <= 0 || (out_ids && (!pos || out_stride <= 0))) return GSDLQ_ERR_INVALID;
  argmax_rows_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>(logits, n, ids, pos, out_ids, out_stride);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_attention_decode_batch(const float* q, int q_stride, const uint16_t* k_cache, const uint16_t* v_cache,
                                 size_t seq_stride, float* out, void* work, size_t work_bytes, int layer, const int* pos,
                                 int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq, float sm_scale,
                                 gsdlq_stream_t stream) {
  if (!q || !k_cache || !v_cache || !out || !work || !pos || batch <= 0 || layer < 0 || max_seq <= 0)
    return GSDLQ_ERR_INVALID;
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads) return GSDLQ_ERR_INVALID;
  const int gq = n_heads / n_kv_heads;
  if (head_dim != 64 && head_dim != 128) return GSDLQ_ERR_INVALID;
  if (gq != 1 && gq != 2 && gq != 4 && gq != 6 && gq != 8) return GSDLQ_ERR_INVALID;
  if (seq_stride < (size_t)(layer + 1) * max_seq * n_kv_heads * head_dim) return GSDLQ_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(work)) &
      15u)
    return GSDLQ_ERR_INVALID;
  if ((seq_stride * 2) % 16) return GSDLQ_ERR_INVALID;
  if (q_stride < 0 || (q_stride > 0 && q_stride < n_heads * head_dim)) return GSDLQ_ERR_INVALID;
  if (work_bytes < attention_rows_work(batch, n_heads, head_dim)) return GSDLQ_ERR_INVALID;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // splits of the position range so that about four CTAs per SM are busy (each split at least one tile)
  const int base = batch * n_kv_heads, tiles = (max_seq + 31) / 32;
  int splits = (4 * sms + base - 1) / base;
  splits = std::max(1, std::min(std::min(splits, AT_MAXSPLIT), tiles));
  const dim3 grid(batch, n_kv_heads, splits);
  float* wk = static_cast<float*>(work);
#define GSDLQ_AD(hd, g)                                                                                          \
  attention_decode_kernel<hd, g><<<grid, AD_THREADS, 0, st>>>(q, k_cache, v_cache, seq_stride, out, wk, layer, pos, \
                                                               batch, n_heads, n_kv_heads, max_seq, sm_scale, splits, \
                                                               q_stride)
  if (head_dim == 64) {
    switch (gq) {
      case 1: GSDLQ_AD(64, 1); break;
      case 2: GSDLQ_AD(64, 2); break;
      case 4: GSDLQ_AD(64, 4); break;
      case 6: GSDLQ_AD(64, 6); break;
      default: GSDLQ_AD(64, 8); break;
    }
  } else {
    switch (gq) {
      case 1: GSDLQ_AD(128, 1); break;
      case 2: GSDLQ_AD(128, 2); break;
      case 4: GSDLQ_AD(128, 4); break;
      case 6: GSDLQ_AD(128, 6); break;
      default: GSDLQ_AD(128, 8); break;
    }
  }
#undef GSDLQ_AD
  GSDLQ_CUDA_CHECK_LAUNCH();
  if (splits > 1) {
    attention_combine_kernel<<<dim3(batch, n_heads), head_dim, 0, st>>>(wk, out, batch, n_heads, head_dim, splits);
    GSDLQ_CUDA_CHECK_LAUNCH();
  }
  return GSDLQ_OK;
}

}  // extern "C"

// hexmm.cu -- the batched packed linear: B <= 64 tokens through one GSD-LQ matrix as a dequant-GEMM on
// the tensor cores (the batch-B counterpart of gsd_cpu_lowrank_proj + gsd_cpu_hex2d_matvec,
// gsd_lq_cpu_engine.c:111-183, applied to each token).
//
//   y[b][r] = sum_c W[r][c] x[b][c] + sum_{kinks of r} delta * x[b][col] + sum_j U[r][j] tmp[b][j],
//   W[r][2p + i] = xy[code(r, p)][i] * scale(r, p / 32),  tmp[b][j] = S[j] * (Vt[j] . x[b]).
//
// Layout of the work.  A CTA of 4 warps owns 64 weight rows and a contiguous run of 64-column k-blocks
// (split-K over CTAs, so that enough loads are in flight on every SM).  Per k-block:
//   - each thread decodes 16 code bytes of one row (32 weights, one scale group) through a 256-entry
//     float2 table into fp32 weights, W = xy * scale as the reference's dequant defines them, and writes
//     each as an fp16 hi + lo pair into two shared W tiles (about 22 significant bits together);
//   - the block's activations of every token are written as fp16 hi + lo splits (x scaled per token by a
//     power of two that puts max|x_b| in [2^14, 2^15), so both halves stay normal);
//   - mma.sync m16n8k16 (fp16 in, fp32 accumulate): warp w takes rows 16w..16w+15; per 8-token n-tile
//     and k-step three MMAs, W_hi x_hi + W_hi x_lo + W_lo x_hi (the lo * lo term is below fp32 rounding);
//   - the codes and scales of the block two ahead and the activations of the next block are loaded into
//     registers while this one is computed.
// The partial sums are added into y (zeroed by the entry point) with fp32 atomics, so the summation
// order over the k-runs is not fixed; the kink and low-rank terms are added once per (row, token) by the
// CTA of the run with the token's index modulo the number of runs.
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "common.cuh"

namespace gsdlq {

constexpr int MM_ROWS = 64;        // weight rows per CTA
constexpr int MM_KB = 64;          // columns per k-block: one scale group
constexpr int MM_THREADS = 128;    // 4 warps, 16 rows each
constexpr int MM_MAXB = 64;        // tokens per call
constexpr int MM_XROW = MM_KB + 8; // halves per shared row (padded: conflict-free fragment loads)

__device__ __forceinline__ void mm_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Per token b and chunk of MM_PREP columns: the chunk's max|x_b| into amax[b] (as ordered bits) and its
// part of S[j] * (Vt[j] . x_b) into tmp[16 b + j] (gsd_cpu_lowrank_proj; fp32 atomics, so the summation
// order is not fixed).  Both start at zero.
constexpr int MM_PREP = 1024;
__global__ void __launch_bounds__(256) hexmm_prep(const float* __restrict__ x, int C, const uint16_t* __restrict__ Vt,
                                                  const float* __restrict__ S, int k, unsigned* __restrict__ amax_bits,
                                                  float* __restrict__ tmp) {
  __shared__ float red[8][17];
  const int b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* xb = x + (size_t)b * C;
  const int c1 = min(C, (int)(blockIdx.y + 1) * MM_PREP);
  float amax = 0.f, acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.f;
  for (int c = blockIdx.y * MM_PREP + threadIdx.x; c < c1; c += 256) {
    const float v = xb[c];
    amax = fmaxf(amax, fabsf(v));
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < k) acc[j] = fmaf(h2f(Vt[(size_t)j * C + c]), v, acc[j]);
  }
  amax = warp_max(amax);
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = warp_sum(acc[j]);
  if (lane == 0) {
    red[warp][16] = amax;
#pragma unroll
    for (int j = 0; j < 16; ++j) red[warp][j] = acc[j];
  }
  __syncthreads();
  if (threadIdx.x < 16 && threadIdx.x < k) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
    atomicAdd(tmp + (size_t)b * 16 + threadIdx.x, S[threadIdx.x] * t);
  }
  if (threadIdx.x == 32) {
    float m = 0.f;
    for (int w = 0; w < 8; ++w) m = fmaxf(m, red[w][16]);
    atomicMax(amax_bits + b, __float_as_uint(m));  // non-negative floats order as their bits
  }
}

// the power of two that puts max|x_b| in [2^14, 2^15), so both fp16 halves of x_b stay normal
__device__ __forceinline__ float hexmm_xscale(unsigned amax_bits) {
  const float m = __uint_as_float(amax_bits);
  int e = 0;
  frexpf(m, &e);  // m < 2^e
  e = max(e, -100);
  return (m > 0.f && m <= 3.0e38f) ? ldexpf(1.f, 15 - e) : 1.f;
}

// NB: 8-token n-tiles (tokens padded to 8 NB with zero activations).
template <int NB>
__global__ void __launch_bounds__(MM_THREADS) hexmm_kernel(const float* __restrict__ x, int B,
                                                           const uint8_t* __restrict__ codes,
                                                           const uint16_t* __restrict__ scales,
                                                           const float* __restrict__ xy, int n_pts,
                                                           const uint16_t* __restrict__ U, int k,
                                                           const uint32_t* __restrict__ row_ptr,
                                                           const uint16_t* __restrict__ kcols,
                                                           const float* __restrict__ kdel, float* __restrict__ y,
                                                           int R, int C, int nsplit, const unsigned* __restrict__ amax_bits,
                                                           const float* __restrict__ tmp) {
  constexpr int BP = NB * 8;                        // padded tokens
  constexpr int XE = BP * MM_KB / MM_THREADS;       // activations of a k-block per thread
  __shared__ __align__(16) uint16_t wh[MM_ROWS * MM_XROW];
  __shared__ __align__(16) uint16_t wl[MM_ROWS * MM_XROW];
  __shared__ __align__(16) uint16_t xh[BP * MM_XROW];
  __shared__ __align__(16) uint16_t xl[BP * MM_XROW];
  __shared__ float2 tab[256];
  __shared__ float s_xsc[MM_MAXB];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, q4 = lane & 3;
  const int r0 = blockIdx.x * MM_ROWS;
  const int split = blockIdx.y;
  const int NP = C / 2, G = C / 64, nkb = C / MM_KB;
  const int kb0 = (int)((long long)nkb * split / nsplit), kb1 = (int)((long long)nkb * (split + 1) / nsplit);
  for (int i = tid; i < 256; i += MM_THREADS) tab[i] = i < n_pts ? make_float2(xy[2 * i], xy[2 * i + 1]) : make_float2(0.f, 0.f);
  for (int i = tid; i < BP; i += MM_THREADS) s_xsc[i] = i < B ? hexmm_xscale(amax_bits[i]) : 0.f;
  __syncthreads();

  // this thread's share of a k-block: 16 code bytes (32 weights) of row drow, and XE activations
  const int drow = tid >> 1, dhalf = tid & 1;
  const bool rok = r0 + drow < R;
  const uint8_t* cp = codes + (size_t)(rok ? r0 + drow : 0) * NP + dhalf * 16;
  const uint16_t* scp = scales + (size_t)(rok ? r0 + drow : 0) * G;
  auto load_x = [&](int kb, float (&xr)[XE]) {
#pragma unroll
    for (int i = 0; i < XE; ++i) {
      const int e = tid + i * MM_THREADS, b = e / MM_KB, c = e - b * MM_KB;
      xr[i] = b < B ? x[(size_t)b * C + kb * MM_KB + c] * s_xsc[b] : 0.f;
    }
  };
  // codes and scales two k-blocks ahead (HBM), activations one ahead (L2)
  uint4 cw = make_uint4(0u, 0u, 0u, 0u), cw2 = make_uint4(0u, 0u, 0u, 0u);
  uint16_t sc = 0, sc2 = 0;
  float xr[XE];
  if (kb1 > kb0) {
    if (rok) {
      cw = *reinterpret_cast<const uint4*>(cp + kb0 * 32);
      sc = scp[kb0];
      if (kb0 + 1 < kb1) {
        cw2 = *reinterpret_cast<const uint4*>(cp + (kb0 + 1) * 32);
        sc2 = scp[kb0 + 1];
      }
    }
    load_x(kb0, xr);
  }
  float acc[NB][4];
#pragma unroll
  for (int n = 0; n < NB; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  bool bad = false;
  for (int kb = kb0; kb < kb1; ++kb) {
    // ---- stage block kb: W rows as fp16, activations as fp16 hi + lo ----
    const float s = h2f(sc);
    const uint32_t cv[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int code = (int)((cv[i >> 2] >> (8 * (i & 3))) & 0xffu);
      bad |= rok && code >= n_pts;
      const float2 p = tab[code];
      const float w0 = p.x * s, w1 = p.y * s;  // a3 dequant: one fp32 multiply per weight
      const uint16_t h0 = f2h(w0), h1 = f2h(w1);
      const int o = drow * MM_XROW + dhalf * 32 + 2 * i;
      *reinterpret_cast<uint32_t*>(wh + o) = (uint32_t)h0 | ((uint32_t)h1 << 16);
      *reinterpret_cast<uint32_t*>(wl + o) = (uint32_t)f2h(w0 - h2f(h0)) | ((uint32_t)f2h(w1 - h2f(h1)) << 16);
    }
#pragma unroll
    for (int i = 0; i < XE; ++i) {
      const int e = tid + i * MM_THREADS, b = e / MM_KB, c = e - b * MM_KB;
      const uint16_t hi = f2h(xr[i]);
      xh[b * MM_XROW + c] = hi;
      xl[b * MM_XROW + c] = f2h(xr[i] - h2f(hi));
    }
    // ---- the next block's operands into registers while this one is multiplied ----
    cw = cw2;
    sc = sc2;
    if (rok && kb + 2 < kb1) {
      cw2 = *reinterpret_cast<const uint4*>(cp + (kb + 2) * 32);
      sc2 = scp[kb + 2];
    }
    if (kb + 1 < kb1) load_x(kb + 1, xr);
    __syncthreads();
    const int ao = (16 * warp + g) * MM_XROW + 2 * q4;
#pragma unroll
    for (int kk = 0; kk < MM_KB / 16; ++kk) {
      uint32_t ah[4], al[4];
      const int o = ao + kk * 16;
      ah[0] = *reinterpret_cast<const uint32_t*>(wh + o);
      ah[1] = *reinterpret_cast<const uint32_t*>(wh + o + 8 * MM_XROW);
      ah[2] = *reinterpret_cast<const uint32_t*>(wh + o + 8);
      ah[3] = *reinterpret_cast<const uint32_t*>(wh + o + 8 * MM_XROW + 8);
      al[0] = *reinterpret_cast<const uint32_t*>(wl + o);
      al[1] = *reinterpret_cast<const uint32_t*>(wl + o + 8 * MM_XROW);
      al[2] = *reinterpret_cast<const uint32_t*>(wl + o + 8);
      al[3] = *reinterpret_cast<const uint32_t*>(wl + o + 8 * MM_XROW + 8);
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const uint16_t* bh = xh + (n * 8 + g) * MM_XROW + kk * 16 + 2 * q4;
        const uint16_t* bl = xl + (n * 8 + g) * MM_XROW + kk * 16 + 2 * q4;
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(bh), bh1 = *reinterpret_cast<const uint32_t*>(bh + 8);
        mm_f16_16816(acc[n], ah, bh0, bh1);
        mm_f16_16816(acc[n], ah, *reinterpret_cast<const uint32_t*>(bl), *reinterpret_cast<const uint32_t*>(bl + 8));
        mm_f16_16816(acc[n], al, bh0, bh1);
      }
    }
    __syncthreads();  // every read of the tiles is done before the next block is staged
  }
  if (bad) raise_flag(GSDLQ_FLAG_BAD_CODE);
  // ---- this run's partial sums into y (unscaled): lane (g, q4) holds rows g, g+8, tokens 2q4, 2q4+1 ----
  if (kb1 > kb0) {
#pragma unroll
    for (int n = 0; n < NB; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = r0 + 16 * warp + g + (e >= 2 ? 8 : 0), b = n * 8 + 2 * q4 + (e & 1);
        if (r < R && b < B) atomicAdd(y + (size_t)b * R + r, acc[n][e] / s_xsc[b]);
      }
    }
  }
  // ---- kinks and the low-rank term, once per (row, token): tokens b = split (mod nsplit) ----
  bool badk = false;
  for (int i = tid; i < MM_ROWS * BP; i += MM_THREADS) {
    const int rr = i / BP, b = i - rr * BP, r = r0 + rr;
    if (r >= R || b >= B || b % nsplit != split) continue;
    float v = 0.f;
    for (int j = 0; j < k; ++j) v = fmaf(h2f(U[(size_t)r * k + j]), tmp[(size_t)b * 16 + j], v);
    const float* xb = x + (size_t)b * C;
    for (uint32_t e = row_ptr[r]; e < row_ptr[r + 1]; ++e) {
      const int col = kcols[e];
      if (col < C) v = fmaf(kdel[e], xb[col], v);
      else badk = true;
    }
    atomicAdd(y + (size_t)b * R + r, v);
  }
  if (badk) raise_flag(GSDLQ_FLAG_BAD_KINK);
}

template <int NB>
static cudaError_t hexmm_launch_nb(dim3 grid, cudaStream_t s, const float* x, int B, const uint8_t* codes,
                                   const uint16_t* scales, const float* xy, int n_pts, const uint16_t* U, int k,
                                   const uint32_t* rp, const uint16_t* kc, const float* kd, float* y, int R, int C,
                                   int nsplit, const unsigned* amax, const float* tmp) {
  hexmm_kernel<NB><<<grid, MM_THREADS, 0, s>>>(x, B, codes, scales, xy, n_pts, U, k, rp, kc, kd, y, R, C, nsplit, amax, tmp);
  return cudaGetLastError();
}

int num_sms();
int record_cuda_error(cudaError_t e);

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_hex2d_matmul(const float* x, int batch, const uint8_t* codes, const uint16_t* scales,
                                  const float* xy_table, const uint16_t* U, const float* S, const uint16_t* Vt,
                                  const uint32_t* kink_row_ptr, const uint16_t* kink_cols, const float* kink_deltas,
                                  float* y, float* work, int rows, int cols, int k_dim, int n_pts, gsdlq_stream_t stream) {
  if (!x || !codes || !scales || !xy_table || !kink_row_ptr || !y || !work) return GSDLQ_ERR_INVALID;
  if (batch < 1 || batch > MM_MAXB || rows <= 0 || cols <= 0 || cols % 64 != 0 || cols > 65535) return GSDLQ_ERR_INVALID;
  if (k_dim < 0 || k_dim > 16 || (k_dim > 0 && (!U || !S || !Vt))) return GSDLQ_ERR_INVALID;
  if (n_pts < 1 || n_pts > 256) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(codes) & 15u) return GSDLQ_ERR_INVALID;  // 16-byte code loads
  if ((reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(U) | reinterpret_cast<uintptr_t>(Vt)) & 1u)
    return GSDLQ_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(work)) & 3u)
    return GSDLQ_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* amax = reinterpret_cast<unsigned*>(work);  // per-token max|x| (bits)
  float* tmp = work + MM_MAXB;
  cudaError_t e = cudaMemsetAsync(y, 0, sizeof(float) * (size_t)batch * rows, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(work, 0, sizeof(float) * 17 * MM_MAXB, s);
  if (e != cudaSuccess) return record_cuda_error(e);
  hexmm_prep<<<dim3(batch, (cols + MM_PREP - 1) / MM_PREP), 256, 0, s>>>(x, cols, Vt, S, k_dim, amax, tmp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return record_cuda_error(e);
  // k-runs per row tile: about eight CTAs per SM in all up to 16 tokens (shorter load chains per CTA),
  // four above (the wide-batch kernels hold more registers), at least one k-block each
  const int tiles = (rows + MM_ROWS - 1) / MM_ROWS, nkb = cols / MM_KB;
  const int per_sm = batch <= 16 ? 8 : 4;
  const int nsplit = std::max(1, std::min(nkb, (per_sm * num_sms() + tiles - 1) / tiles));
  const dim3 grid(tiles, nsplit);
  const float* kd = kink_deltas;
  switch ((batch + 7) / 8) {
    case 1: e = hexmm_launch_nb<1>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
    case 2: e = hexmm_launch_nb<2>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
    case 3: e = hexmm_launch_nb<3>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
    case 4: e = hexmm_launch_nb<4>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
    case 5: e = hexmm_launch_nb<5>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
    case 6: e = hexmm_launch_nb<6>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
    case 7: e = hexmm_launch_nb<7>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
    default: e = hexmm_launch_nb<8>(grid, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, kd, y, rows, cols, nsplit, amax, tmp); break;
  }
  if (e != cudaSuccess) return record_cuda_error(e);
  return GSDLQ_OK;
}

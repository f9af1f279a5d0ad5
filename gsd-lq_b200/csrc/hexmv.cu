// hexmv.cu -- fused GSD-LQ packed linear for batch-1 decode on sm_100a.
//
// Computes, for every row r of up to three packed matrices that share one input x,
//   y[r] = sum_p xy[code(r,p)] . (x[2p], x[2p+1]) * scale(r, p/32)      (lattice part)
//        + sum_{kinks of r} delta * x[col]                               (CSR kinks)
//        + sum_j U[r,j] * tmp_k[j],  tmp_k[j] = S[j] * (Vt[j] . x)        (low rank)
// -- the reference's gsd_cpu_lowrank_proj + gsd_cpu_hex2d_matvec pair
// (gsd_lq_v2/gsd_lq_cpu_engine.c:111-183) -- in ONE kernel, with the input
// transform (RMSNorm, embedding lookup) fused into the prologue and the
// consumer of y (residual add, SwiGLU, RoPE + fp16 KV-cache append, greedy
// argmax) fused into the epilogue.
//
// Arithmetic.  An A2 lattice point is (r0 + r1/2, r1*sqrt3/2) with small
// integers r0, r1, so
//     xy . (x0, x1) = r0 * x0 + r1 * (x0/2 + sqrt3/2 * x1) = r0 * a + r1 * b.
// (r0, r1) are exact in bf16; (a, b) is split into bf16 hi + lo parts (about 16
// mantissa bits together).  One warp-level mma.sync m16n8k16 then computes, for
// 16 rows x 8 code pairs, the hi and lo dot products in B columns 0 and 1 with
// fp32 accumulation.  The tensor core only does the multiply-adds; the kernel
// is HBM-bound on the code stream (0.53 B/weight).
//
// Decode.  A code byte becomes its bf16x2 (r0, r1) through one byte-permute
// (PRMT: code -> bits 8..15, lane*4 -> bits 0..7) and one 32-bit shared load
// from a 256-entry table replicated once per lane in the lane's own bank
// (entry c of lane l at byte c*256 + l*4), so the 32 lookups of a warp never
// conflict.
//
// Work split.  A CTA (8 warps) owns whole 16-row strips: every warp covers a
// contiguous range of 64-column scale groups of the strip, partial row sums
// meet in shared memory, and the epilogue sees complete rows.  CTAs are
// persistent (grid <= resident capacity) so that the table build and the
// input staging are paid once per CTA.  The low-rank projections are computed
// by the first CTAs to start (an atomic ticket) and published through a
// counter that the epilogues wait on with a bounded spin.
#include <algorithm>
#include <cstdio>

#include "common.cuh"

namespace gsdlq {

constexpr int HX_WARPS = 8;
constexpr int HX_THREADS = HX_WARPS * kWarp;
constexpr int HX_TAB_BYTES = 256 * 256;
constexpr int HX_PF = 4;  // groups of codes kept in flight per warp

struct HexmvParams {
  gsdlq_linear_job_t job;
  const float* xy_table;     // drop-in path: decode table derived from this float table
  const float* tmp_k_ext;    // drop-in path: caller-computed tmp_k for mat[0]
  int n_pts;
  int cols;
  int units;
  int unit_begin[4];         // prefix sums of strips per matrix (non-pair modes)
  int n_lowrank_jobs;
  int pair;                  // SWIGLU: mat[0], mat[1] processed strip by strip together
};

struct HexmvSmem {
  int cols;
  __device__ __forceinline__ float* xf(uint8_t* base) const { return reinterpret_cast<float*>(base + HX_TAB_BYTES); }
  __device__ __forceinline__ uint32_t* xs_hi(uint8_t* base) const { return reinterpret_cast<uint32_t*>(xf(base) + cols); }
  __device__ __forceinline__ uint32_t* xs_lo(uint8_t* base) const { return xs_hi(base) + cols / 2; }
  __device__ __forceinline__ float* scl(uint8_t* base) const { return reinterpret_cast<float*>(xs_lo(base) + cols / 2); }
  // scale rows: 2 matrices x 16 rows x (G + 1) floats (row padded by one word)
  __device__ __forceinline__ float* red(uint8_t* base) const { return scl(base) + 2 * 16 * (cols / 64 + 1); }
  __device__ __forceinline__ float* misc(uint8_t* base) const { return red(base) + HX_WARPS * 32; }
};

inline size_t hexmv_smem_bytes(int cols) {
  const size_t g = cols / 64;
  return HX_TAB_BYTES + 4ull * cols /*xf*/ + 4ull * cols /*xs hi+lo*/ + 4ull * 2 * 16 * (g + 1) +
         4ull * HX_WARPS * 32 + 4ull * (8 + 3 * 16 + 8);
}

// (r0, r1) of code c in the radius-R enumeration (r0 outer, r1 inner, |r0+r1| <= R).
__device__ __forceinline__ bool lattice_of_code(int c, int R, int& r0, int& r1) {
  for (int a = -R; a <= R; ++a) {
    const int lo = max(-R, -R - a), hi = min(R, R - a);
    const int n = hi - lo + 1;
    if (c < n) {
      r0 = a;
      r1 = lo + c;
      return true;
    }
    c -= n;
  }
  return false;
}

__device__ void build_decode_table(uint8_t* smem, const HexmvParams& P) {
  const int R = P.job.mat[0].radius;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    int r0 = 0, r1 = 0;
    bool ok;
    if (P.xy_table != nullptr) {
      ok = i < P.n_pts;
      if (ok) {
        const float x = P.xy_table[2 * i], y = P.xy_table[2 * i + 1];
        const float rf1 = rintf(y * 1.1547005383792515f);
        const float rf0 = x - 0.5f * rf1;
        r0 = (int)rf0;
        r1 = (int)rf1;
        const float yy = (float)((double)r1 * 0.8660254037844386);
        if ((float)r0 != rf0 || yy != y || fabsf(rf0) > 16.f || fabsf(rf1) > 16.f) {
          raise_flag(GSDLQ_FLAG_BAD_TABLE);
          r0 = r1 = 0;
        }
      }
    } else {
      ok = lattice_of_code(i, R, r0, r1);
    }
    if (!ok) r0 = r1 = 0;
    const uint32_t e = pack_bf16x2((float)r0, (float)r1);
    uint4 v = make_uint4(e, e, e, e);
    uint4* row = reinterpret_cast<uint4*>(smem + i * 256);
#pragma unroll
    for (int w = 0; w < 8; ++w) row[w] = v;
  }
}

// Input staging: xf = transformed fp32 input, xs_hi/xs_lo = bf16 splits of (a, b).
__device__ void stage_input(uint8_t* smem, const HexmvSmem& L, const HexmvParams& P) {
  const gsdlq_linear_job_t& J = P.job;
  const int C = P.cols;
  float* xf = L.xf(smem);
  float* misc = L.misc(smem);
  const int tid = threadIdx.x;
  // 1. raw row into xf
  if (J.input_mode == GSDLQ_IN_EMBED) {
    int tok = *J.token;
    if (tok < 0 || tok >= J.vocab) {
      if (tid == 0) raise_flag(GSDLQ_FLAG_BAD_TOKEN);
      tok = 0;
    }
    const uint16_t* row = J.embed + (size_t)tok * C;
    for (int c = tid; c < C; c += blockDim.x) {
      const float v = h2f(row[c]);
      xf[c] = v;
      if (blockIdx.x == 0 && J.x_out != nullptr) J.x_out[c] = v;
    }
  } else {
    const float2* x2 = reinterpret_cast<const float2*>(J.x);
    float2* xf2 = reinterpret_cast<float2*>(xf);
    for (int p = tid; p < C / 2; p += blockDim.x) xf2[p] = x2[p];
  }
  __syncthreads();
  // 2. RMSNorm: out = x * (1/sqrt(sum(x^2)/C + eps)) * w   (gsd_lq_cpu_engine.c:67-82)
  if (J.input_mode != GSDLQ_IN_PLAIN) {
    float ss = 0.f;
    for (int c = tid; c < C; c += blockDim.x) ss += xf[c] * xf[c];
    ss = warp_sum(ss);
    float* red = L.red(smem);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
      misc[0] = 1.0f / sqrtf(t / (float)C + J.eps);
    }
    __syncthreads();
    const float inv = misc[0];
    for (int c = tid; c < C; c += blockDim.x) xf[c] = __fmul_rn(__fmul_rn(xf[c], inv), J.norm_w[c]);
    __syncthreads();
  }
  // 3. (a, b) = (x0, x0/2 + sqrt3/2 * x1) split into bf16 hi + lo
  uint32_t* hi = L.xs_hi(smem);
  uint32_t* lo = L.xs_lo(smem);
  for (int p = tid; p < C / 2; p += blockDim.x) {
    const float x0 = xf[2 * p], x1 = xf[2 * p + 1];
    const float a = x0;
    const float b = fmaf(0.8660254037844386f, x1, 0.5f * x0);
    uint32_t h, l;
    split_bf16x2(a, b, h, l);
    hi[p] = h;
    lo[p] = l;
  }
}

__device__ __forceinline__ uint32_t tab_lookup(const uint8_t* smem, uint32_t word, uint32_t lane4, uint32_t sel) {
  const uint32_t off = __byte_perm(word, lane4, sel);
  return *reinterpret_cast<const uint32_t*>(smem + off);
}

// One 64-column scale group of one 16-row strip: 4 MMAs; returns hi+lo sums for rows g, g+8.
__device__ __forceinline__ void group_mma(const uint8_t* smem, uint2 ca, uint2 cb, const uint32_t (&bq)[8],
                                          uint32_t lane4, float& r_g, float& r_h) {
  float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t wa = (j < 2) ? ca.x : ca.y;
    const uint32_t wb = (j < 2) ? cb.x : cb.y;
    const uint32_t k0 = 2 * (j & 1);
    const uint32_t s0 = 0x5504u | (k0 << 4), s1 = 0x5504u | ((k0 + 1) << 4);
    uint32_t a[4];
    a[0] = tab_lookup(smem, wa, lane4, s0);  // row g,   pair 8q+2j
    a[1] = tab_lookup(smem, wb, lane4, s0);  // row g+8, pair 8q+2j
    a[2] = tab_lookup(smem, wa, lane4, s1);  // row g,   pair 8q+2j+1
    a[3] = tab_lookup(smem, wb, lane4, s1);  // row g+8, pair 8q+2j+1
    mma_bf16_16816(d, a, bq[2 * j], bq[2 * j + 1], d);
  }
  r_g = d[0] + d[1];
  r_h = d[2] + d[3];
}

// Block-wide dot of xf with one fp16 row of length C (for the low-rank projection).
__device__ float block_dot_f16(const float* xf, const uint16_t* v, int C, float* red) {
  float s = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) s += xf[c] * h2f(v[c]);
  s = warp_sum(s);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  __syncthreads();
  return t;
}

template <int EPI>
__global__ void __launch_bounds__(HX_THREADS, 1) hexmv_kernel(const __grid_constant__ HexmvParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const gsdlq_linear_job_t& J = P.job;
  const HexmvSmem L{P.cols};
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gl = lane >> 2, q = lane & 3;
  const int C = P.cols, G = C / 64, NP = C / 2;
  float* misc = L.misc(smem);
  float* s_tmpk = misc + 8;              // [3][16]
  int* s_flags = reinterpret_cast<int*>(misc + 8 + 48);  // [0]: ticket, [1]: tmpk ready
  unsigned int* ws = J.workspace;

  build_decode_table(smem, P);
  stage_input(smem, L, P);
  if (tid == 0) s_flags[1] = 0;
  __syncthreads();

  // ---- low-rank producers: first CTAs to arrive compute tmp_k[m][j] --------------------
  if (P.n_lowrank_jobs > 0) {
    while (true) {
      if (tid == 0) s_flags[0] = (int)atomicAdd(&ws[0], 1u);
      __syncthreads();
      const int t = s_flags[0];
      __syncthreads();
      if (t >= P.n_lowrank_jobs) break;
      int m = 0, j = t;
      while (m < P.job.n_mat - 1 && j >= J.mat[m].k_dim) j -= J.mat[m].k_dim, ++m;
      const gsdlq_hexmat_t& M = J.mat[m];
      const float dot = block_dot_f16(L.xf(smem), M.Vt + (size_t)j * C, C, L.red(smem));
      if (tid == 0) {
        reinterpret_cast<volatile float*>(ws)[16 + m * 16 + j] = dot * M.S[j];
        __threadfence();
        atomicAdd(&ws[1], 1u);
      }
    }
  }

  const uint32_t lane4 = (uint32_t)lane * 4u;
  const uint32_t* xs_hi = L.xs_hi(smem);
  const uint32_t* xs_lo = L.xs_lo(smem);
  float* scl = L.scl(smem);
  float* red = L.red(smem);
  const int nmat_unit = P.pair ? 2 : 1;

  // this warp's range of scale groups
  const int g_begin = (warp * G) / HX_WARPS, g_end = ((warp + 1) * G) / HX_WARPS;

  for (int u = blockIdx.x; u < P.units; u += gridDim.x) {
    int m0 = 0, strip = u;
    if (!P.pair) {
      while (m0 < J.n_mat - 1 && u >= P.unit_begin[m0 + 1]) ++m0;
      strip = u - P.unit_begin[m0];
    }
    const int rbase = strip * 16;
    // stage this strip's scales (fp16 -> fp32) for the 1 or 2 matrices of the unit
    for (int mm = 0; mm < nmat_unit; ++mm) {
      const gsdlq_hexmat_t& M = J.mat[m0 + mm];
      for (int i = tid; i < 16 * G; i += blockDim.x) {
        const int rr = i / G, gg = i - rr * G;
        const int row = min(rbase + rr, M.rows - 1);
        scl[(mm * 16 + rr) * (G + 1) + gg] = h2f(M.scales[(size_t)row * G + gg]);
      }
    }
    __syncthreads();

    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int mm = 0; mm < nmat_unit; ++mm) {
      const gsdlq_hexmat_t& M = J.mat[m0 + mm];
      const int ra = min(rbase + gl, M.rows - 1), rb = min(rbase + gl + 8, M.rows - 1);
      const uint8_t* pa = M.codes + (size_t)ra * NP + q * 8;
      const uint8_t* pb = M.codes + (size_t)rb * NP + q * 8;
      const float* sa = scl + (mm * 16 + gl) * (G + 1);
      const float* sb = scl + (mm * 16 + gl + 8) * (G + 1);
      uint2 ca[HX_PF], cb[HX_PF];
#pragma unroll
      for (int i = 0; i < HX_PF; ++i) {
        if (g_begin + i < g_end) {
          ca[i] = ldg_stream_u2(pa + (size_t)(g_begin + i) * 32);
          cb[i] = ldg_stream_u2(pb + (size_t)(g_begin + i) * 32);
        }
      }
      float accg = 0.f, acch = 0.f;
      for (int g = g_begin; g < g_end; g += HX_PF) {
#pragma unroll
        for (int i = 0; i < HX_PF; ++i) {
          const int gg = g + i;
          if (gg < g_end) {
            const uint2 a = ca[i], b = cb[i];
            const int gn = gg + HX_PF;
            if (gn < g_end) {
              ca[i] = ldg_stream_u2(pa + (size_t)gn * 32);
              cb[i] = ldg_stream_u2(pb + (size_t)gn * 32);
            }
            uint32_t bq[8];
            if (gl < 2) {
              const uint4* src = reinterpret_cast<const uint4*>((gl == 0 ? xs_hi : xs_lo) + gg * 32 + q * 8);
              const uint4 v0 = src[0], v1 = src[1];
              bq[0] = v0.x; bq[1] = v0.y; bq[2] = v0.z; bq[3] = v0.w;
              bq[4] = v1.x; bq[5] = v1.y; bq[6] = v1.z; bq[7] = v1.w;
            } else {
#pragma unroll
              for (int t = 0; t < 8; ++t) bq[t] = 0u;
            }
            float rg, rh;
            group_mma(smem, a, b, bq, lane4, rg, rh);
            accg = fmaf(sa[gg], rg, accg);
            acch = fmaf(sb[gg], rh, acch);
          }
        }
      }
      acc[mm][0] = accg;
      acc[mm][1] = acch;
    }
    // lanes q == 0 hold the rows' sums (B columns 2..7 are zero)
    if (q == 0) {
      for (int mm = 0; mm < nmat_unit; ++mm) {
        red[warp * 32 + mm * 16 + gl] = acc[mm][0];
        red[warp * 32 + mm * 16 + gl + 8] = acc[mm][1];
      }
    }
    __syncthreads();

    // ---- epilogue: warp w finishes rows 2w and 2w+1 of each matrix of the unit -------
    const bool need_lr = (P.tmp_k_ext == nullptr) && P.n_lowrank_jobs > 0;
    if (need_lr && s_flags[1] == 0) {
      if (tid == 0) {
        wait_counter_geq(&ws[1], (unsigned)P.n_lowrank_jobs, 1000000000ull);  // 1 s bound
        __threadfence();
      }
      __syncthreads();
      for (int i = tid; i < 48; i += blockDim.x) s_tmpk[i] = reinterpret_cast<volatile float*>(ws)[16 + i];
      if (tid == 0) s_flags[1] = 1;
      __syncthreads();
    }
    float vals[2][2];
    for (int mm = 0; mm < nmat_unit; ++mm) {
      const int m = m0 + mm;
      const gsdlq_hexmat_t& M = J.mat[m];
      for (int k = 0; k < 2; ++k) {
        const int ri = 2 * warp + k;
        const int row = rbase + ri;
        float v = 0.f;
        if (row < M.rows) {
          // kinks of this row, spread over the lanes
          const uint32_t e0 = M.row_ptr[row], e1 = M.row_ptr[row + 1];
          const float* xf = L.xf(smem);
          for (uint32_t e = e0 + lane; e < e1; e += 32) {
            const int col = M.kink_cols[e];
            if (col < C) v += M.kink_deltas[e] * xf[col];
            else raise_flag(GSDLQ_FLAG_BAD_KINK);
          }
          if (M.k_dim > 0 && lane < M.k_dim) {
            const float tk = P.tmp_k_ext ? P.tmp_k_ext[lane] : s_tmpk[m * 16 + lane];
            v += h2f(M.U[(size_t)row * M.k_dim + lane]) * tk;
          }
        }
        v = warp_sum(v);
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < HX_WARPS; ++w) s += red[w * 32 + mm * 16 + ri];
        vals[mm][k] = s + v;
      }
    }
    if (lane == 0) {
      const int r0 = rbase + 2 * warp;
      if constexpr (EPI == GSDLQ_EPI_STORE) {
        const gsdlq_hexmat_t& M = J.mat[m0];
        for (int k = 0; k < 2; ++k) {
          const int row = r0 + k;
          if (row < M.rows) {
            J.y[m0][row] = vals[0][k];
            if (J.argmax_key)
              atomicMax(J.argmax_key, argmax_key(vals[0][k], (uint32_t)(row + J.argmax_index_base)));
          }
        }
      } else if constexpr (EPI == GSDLQ_EPI_RESID) {
        const gsdlq_hexmat_t& M = J.mat[0];
        for (int k = 0; k < 2; ++k) {
          const int row = r0 + k;
          if (row < M.rows) J.y[0][row] = J.resid[row] + vals[0][k];
        }
      } else if constexpr (EPI == GSDLQ_EPI_SWIGLU) {
        const gsdlq_hexmat_t& M = J.mat[0];
        for (int k = 0; k < 2; ++k) {
          const int row = r0 + k;
          if (row < M.rows) {
            const float g = vals[0][k], up = vals[1][k];
            J.y[0][row] = (g / (1.0f + expf(-g))) * up;
          }
        }
      } else if constexpr (EPI == GSDLQ_EPI_ROPE_KV) {
        // rows (r0, r0+1) are one interleaved RoPE pair of one head
        const gsdlq_hexmat_t& M = J.mat[m0];
        if (r0 + 1 < M.rows) {
          const int pos = *J.pos;
          const int hd = J.head_dim;
          const int i = (r0 % hd) >> 1;
          const float v0 = vals[0][0], v1 = vals[0][1];
          const bool pos_ok = pos >= 0 && pos < J.max_seq;
          if (!pos_ok) raise_flag(GSDLQ_FLAG_BAD_POS);
          if (m0 == 2) {  // V: store unrotated
            if (J.y[2]) { J.y[2][r0] = v0; J.y[2][r0 + 1] = v1; }
            if (pos_ok) {
              uint16_t* dst = J.v_cache + ((size_t)J.layer * J.max_seq + pos) * M.rows + r0;
              dst[0] = f2h(v0);
              dst[1] = f2h(v1);
            }
          } else {
            const float2 cs = pos_ok ? reinterpret_cast<const float2*>(J.rope_cs)[(size_t)pos * (hd / 2) + i]
                                     : make_float2(1.f, 0.f);
            const float o0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
            const float o1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
            if (m0 == 0) {
              J.y[0][r0] = o0;
              J.y[0][r0 + 1] = o1;
            } else {
              if (J.y[1]) { J.y[1][r0] = o0; J.y[1][r0 + 1] = o1; }
              if (pos_ok) {
                uint16_t* dst = J.k_cache + ((size_t)J.layer * J.max_seq + pos) * M.rows + r0;
                dst[0] = f2h(o0);
                dst[1] = f2h(o1);
              }
            }
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- the last CTA leaves the workspace counters at zero for the next launch ----------
  if (P.n_lowrank_jobs > 0 && tid == 0) {
    __threadfence();
    if (atomicAdd(&ws[2], 1u) == gridDim.x - 1) {
      for (int i = 0; i < GSDLQ_LINEAR_WS_WORDS; ++i) ws[i] = 0u;  // counters and published tmp_k
      __threadfence();
    }
  }
}

// ---- host side ------------------------------------------------------------------------
static int hexmv_validate_mat(const gsdlq_hexmat_t& M, int cols) {
  if (!M.codes || !M.scales || !M.row_ptr) return GSDLQ_ERR_INVALID;
  // codes are read 8 bytes at a time from row starts (cols/2 is a multiple of 32)
  if (reinterpret_cast<uintptr_t>(M.codes) & 7u) return GSDLQ_ERR_INVALID;
  if (M.rows <= 0 || M.cols != cols || cols <= 0 || cols % 64 != 0) return GSDLQ_ERR_INVALID;
  if (M.k_dim < 0 || M.k_dim > 16) return GSDLQ_ERR_INVALID;
  if (M.k_dim > 0 && (!M.U || !M.S || !M.Vt)) return GSDLQ_ERR_INVALID;
  if (M.radius != 6 && M.radius != 8) return GSDLQ_ERR_INVALID;
  return GSDLQ_OK;
}

// Resident CTAs per SM for a given dynamic smem size, from the hardware limits (no runtime
// occupancy query on the launch path): 228 KB of shared memory per SM with 1 KB reserved per CTA,
// 64K registers per SM at <= 128 registers per thread (ptxas reports 123-128 for hexmv_kernel).
static int hexmv_ctas_per_sm(size_t smem) {
  const size_t per_cta = smem + 1024;
  int by_smem = (int)((228u * 1024u) / per_cta);
  const int by_regs = 65536 / (HX_THREADS * 128);
  return std::max(0, std::min(by_smem, by_regs));
}

template <int EPI>
static int hexmv_launch_t(const HexmvParams& P, cudaStream_t s) {
  const size_t smem = hexmv_smem_bytes(P.cols);
  static int configured_max[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if ((int)smem > configured_max[dev]) {
    cudaError_t e = cudaFuncSetAttribute(hexmv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return record_cuda_error(e);
    configured_max[dev] = 227 * 1024;
  }
  const int per_sm = hexmv_ctas_per_sm(smem);
  if (per_sm < 1) return GSDLQ_ERR_UNSUPPORTED;
  const int grid = std::max(1, std::min(P.units, per_sm * num_sms()));
  hexmv_kernel<EPI><<<grid, HX_THREADS, smem, s>>>(P);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int hexmv_launch(HexmvParams& P, cudaStream_t s) {
  const gsdlq_linear_job_t& J = P.job;
  if (J.n_mat < 1 || J.n_mat > 3) return GSDLQ_ERR_INVALID;
  const int C = J.mat[0].cols;
  P.cols = C;
  if ((size_t)hexmv_smem_bytes(C) > 227 * 1024) return GSDLQ_ERR_UNSUPPORTED;
  for (int m = 0; m < J.n_mat; ++m) {
    const int st = hexmv_validate_mat(J.mat[m], C);
    if (st != GSDLQ_OK) return st;
    if (J.mat[m].radius != J.mat[0].radius) return GSDLQ_ERR_INVALID;
  }
  if (J.input_mode == GSDLQ_IN_PLAIN && !J.x) return GSDLQ_ERR_INVALID;
  if (J.input_mode != GSDLQ_IN_EMBED && (reinterpret_cast<uintptr_t>(J.x) & 7u)) return GSDLQ_ERR_INVALID;  // float2 loads
  if (J.input_mode == GSDLQ_IN_RMSNORM && (!J.x || !J.norm_w)) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_EMBED && (!J.embed || !J.token || !J.norm_w || J.vocab <= 0)) return GSDLQ_ERR_INVALID;
  if (J.input_mode < 0 || J.input_mode > 2) return GSDLQ_ERR_INVALID;
  int lr = 0;
  for (int m = 0; m < J.n_mat; ++m) lr += J.mat[m].k_dim;
  P.n_lowrank_jobs = P.tmp_k_ext ? 0 : lr;
  if (P.n_lowrank_jobs > 0 && !J.workspace) return GSDLQ_ERR_INVALID;
  P.pair = 0;
  P.unit_begin[0] = 0;
  for (int m = 0; m < J.n_mat; ++m) P.unit_begin[m + 1] = P.unit_begin[m] + (J.mat[m].rows + 15) / 16;
  P.units = P.unit_begin[J.n_mat];
  switch (J.epilogue) {
    case GSDLQ_EPI_STORE:
      if (J.n_mat != 1 && J.argmax_key) return GSDLQ_ERR_INVALID;
      for (int m = 0; m < J.n_mat; ++m)
        if (!J.y[m]) return GSDLQ_ERR_INVALID;
      return hexmv_launch_t<GSDLQ_EPI_STORE>(P, s);
    case GSDLQ_EPI_RESID:
      if (J.n_mat != 1 || !J.y[0] || !J.resid) return GSDLQ_ERR_INVALID;
      return hexmv_launch_t<GSDLQ_EPI_RESID>(P, s);
    case GSDLQ_EPI_SWIGLU:
      if (J.n_mat != 2 || !J.y[0] || J.mat[0].rows != J.mat[1].rows) return GSDLQ_ERR_INVALID;
      P.pair = 1;
      P.units = (J.mat[0].rows + 15) / 16;
      return hexmv_launch_t<GSDLQ_EPI_SWIGLU>(P, s);
    case GSDLQ_EPI_ROPE_KV:
      if (J.n_mat != 3 || !J.y[0] || !J.k_cache || !J.v_cache || !J.pos || !J.rope_cs) return GSDLQ_ERR_INVALID;
      if (J.interleaved != 1 || J.head_dim <= 0 || J.head_dim % 16 != 0 || J.max_seq <= 0) return GSDLQ_ERR_UNSUPPORTED;
      if (J.mat[1].rows != J.mat[2].rows || J.mat[0].rows % J.head_dim || J.mat[1].rows % J.head_dim)
        return GSDLQ_ERR_INVALID;
      return hexmv_launch_t<GSDLQ_EPI_ROPE_KV>(P, s);
    default:
      return GSDLQ_ERR_INVALID;
  }
}

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_linear(const gsdlq_linear_job_t* job, gsdlq_stream_t stream) {
  if (!job) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  P.job = *job;
  return hexmv_launch(P, static_cast<cudaStream_t>(stream));
}

extern "C" int gsdlq_hex2d_matvec(const float* x, const uint8_t* codes, const uint16_t* scales, const float* xy_table,
                                  const uint16_t* U, const float* tmp_k, const uint32_t* kink_row_ptr,
                                  const uint16_t* kink_cols, const float* kink_deltas, float* y, int rows, int cols,
                                  int k_dim, int n_pts, gsdlq_stream_t stream) {
  if (!x || !codes || !scales || !xy_table || !kink_row_ptr || !y) return GSDLQ_ERR_INVALID;
  if (n_pts <= 0 || n_pts > 256) return GSDLQ_ERR_INVALID;
  if (k_dim > 0 && (!U || !tmp_k)) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  gsdlq_linear_job_t& J = P.job;
  J.n_mat = 1;
  gsdlq_hexmat_t& M = J.mat[0];
  M.codes = codes;
  M.scales = scales;
  M.U = U;
  M.S = nullptr;
  M.Vt = nullptr;
  M.row_ptr = kink_row_ptr;
  M.kink_cols = kink_cols;
  M.kink_deltas = kink_deltas;
  M.rows = rows;
  M.cols = cols;
  M.k_dim = k_dim;
  M.radius = 8;  // unused when xy_table is given
  J.input_mode = GSDLQ_IN_PLAIN;
  J.x = x;
  J.epilogue = GSDLQ_EPI_STORE;
  J.y[0] = y;
  P.xy_table = xy_table;
  P.n_pts = n_pts;
  P.tmp_k_ext = k_dim > 0 ? tmp_k : nullptr;
  // the drop-in signature carries no S/Vt: the low-rank term comes from tmp_k
  if (k_dim > 0) {
    M.S = tmp_k;   // non-null placeholders so validation passes; never read when tmp_k_ext is set
    M.Vt = U;
  }
  return hexmv_launch(P, static_cast<cudaStream_t>(stream));
}

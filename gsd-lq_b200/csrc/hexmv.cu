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
// conflict.  The other half of every 256-byte table row holds 128 bytes of the
// staged activation splits.
//
// Work split: persistent stream-K.  One CTA per SM: 14 streaming warps and 2
// helper warps.  The (16-row strip, 64-column group) iterations of the launch
// are dealt to the streaming warps as equal contiguous ranges, so every warp
// streams the same number of code bytes.  A unit is UG consecutive 64-column
// groups of one strip; the next unit's codes are always in flight in registers,
// across strip boundaries.  A warp's contribution to a
// strip (a "segment") goes to a per-strip partial slot; a per-strip counter
// tells the warp that completes a strip to sum the slots in slot order
// (deterministic) and run the epilogue.  The helper warps compute the low-rank
// projections (one tmp_k value per ticket) and then each strip's kink and
// low-rank terms into one more slot, off the streaming warps' critical path.
//
// Launch order (programmatic dependent launch): decode table, staged scales
// and the first code prefetches are issued BEFORE griddepcontrol.wait, so they
// overlap the previous kernel; the input x is read only after it.
#include <algorithm>
#include <cstdio>

#include "common.cuh"

namespace gsdlq {

constexpr int HX_WARPS = 16;
constexpr int HX_STREAM = 14;
constexpr int HX_THREADS = HX_WARPS * kWarp;

// control words at the start of the workspace
constexpr int CTL_TK_TICKET = 0;    // low-rank job tickets
constexpr int CTL_TK_DONE = 1;      // low-rank jobs published
constexpr int CTL_KINK_TICKET = 2;  // helper strip tickets
constexpr int CTL_DONE = 3;         // CTAs finished
constexpr int CTL_TMPK = 16;        // 48 floats: tmp_k[m][j]
constexpr int CTL_WORDS = 64;

struct HexmvParams {
  gsdlq_linear_job_t job;
  const float* xy_table;   // drop-in path: decode table derived from this float table
  const float* tmp_k_ext;  // drop-in path: caller-computed tmp_k for mat[0]
  int n_pts;
  int cols, G, NP;
  int n_strips, nmat;      // nmat: matrices per strip unit (2 in SwiGLU pair mode)
  int strip_begin[4];      // prefix of strips per matrix (non-pair modes)
  int UG, GU;              // groups per work unit, units per strip (G = UG * GU)
  long long T;             // iterations (work units) = n_strips * GU
  int W;                   // streaming warps in the launch
  int max_seg;             // partial slots per strip for streaming segments (+1 helper slot)
  int n_lr_jobs;
  int sc_strips;           // capacity of the staged-scale window (strips)
  int ovf_bytes;           // activation-split overflow region
  unsigned* ctl;
  unsigned* cnt;           // [n_strips]
  float* part;             // [n_strips][max_seg + 1][nmat * 16]
};

// ---- partition helpers (identical on host and device) --------------------------------
__host__ __device__ __forceinline__ long long it_begin(int w, long long T, int W) { return (long long)w * T / W; }
// warp whose range contains iteration i: the largest w with it_begin(w) <= i
__host__ __device__ __forceinline__ int warp_of(long long i, long long T, int W) {
  return (int)(((i + 1) * (long long)W - 1) / T);
}

inline size_t hexmv_ws_bytes_for(int n_strips, int max_seg, int nmat) {
  return sizeof(unsigned) * (CTL_WORDS + (size_t)n_strips) +
         sizeof(float) * (size_t)n_strips * (max_seg + 1) * nmat * 16 + 256;
}

// ---- shared memory --------------------------------------------------------------------
// The decode table sits at the absolute shared-window address 0x10000 so that one byte
// permute builds a lookup address from a code byte (bits 8..15), the lane (bits 2..6) and
// the constant 0x01 (bits 16..23).  Dynamic shared memory starts at a small offset B (the
// system-reserved bytes); the buffers below the table use [0, 0x10000 - B):
//   activation-split overflow chunks | staged scale window | misc
// and the fp32 input xf follows the table.  The host sizes the allocation for B <= 4 KB;
// the kernel checks B and raises GSDLQ_FLAG_UNSUPPORTED if the assumption fails.
constexpr uint32_t HX_TAB_ABS = 0x10000u;
constexpr int HX_BASE_MAX = 4096;

struct HxLayout {
  int sc_off, misc_off, low_end;
};

// staged scales: row-major fp16 rows of the CTA's strips, [local strip][matrix][row][sc_words]
// 32-bit words, sc_words = an odd number >= ceil(G/2) so that the 8 rows a warp reads at the
// same column sit in 8 different banks; one 32-bit load gives a row's scales of two groups
__host__ __device__ inline int hx_sc_words(int G) { return ((G + 1) / 2) | 1; }

__host__ __device__ inline HxLayout hx_layout(int ovf_bytes, int sc_strips, int nmat, int G) {
  HxLayout L;
  L.sc_off = ovf_bytes;
  const int sc_bytes = sc_strips * nmat * 16 * hx_sc_words(G) * 4;
  L.misc_off = L.sc_off + ((sc_bytes + 15) & ~15);
  L.low_end = L.misc_off + 64 * 4;
  return L;
}

inline int hx_dyn_smem(int cols) { return (int)(2 * HX_TAB_ABS) + 4 * cols + 64; }

// dynamic-smem offset of the 128-byte activation-split chunk `ch` (chunk 2g = hi words of
// group g, 2g+1 = lo words); the first 256 chunks fill the free halves of the table rows
__device__ __forceinline__ uint32_t xs_chunk(int ch, uint32_t tab_off) {
  return ch < 256 ? tab_off + (uint32_t)ch * 256u + 128u : (uint32_t)(ch - 256) * 128u;
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

__device__ __forceinline__ void build_decode_table(uint8_t* tab, const HexmvParams& P) {
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
    const uint4 v = make_uint4(e, e, e, e);
    uint4* row = reinterpret_cast<uint4*>(tab + i * 256);
#pragma unroll
    for (int w = 0; w < 8; ++w) row[w] = v;
  }
}

// Decode lookup: PRMT assembles the absolute shared address 0x10000 | code << 8 | lane << 2
// (lane4x = lane*4 | 0x0100 supplies bytes 0 and 2), one 32-bit shared load reads the entry.
// The load is not volatile (the table is constant after the prologue barrier), so lookups of
// different k-steps and groups can be scheduled around the MMAs; lane4x is derived from a
// shared-memory read made after that barrier, which keeps every lookup behind it.
__device__ __forceinline__ uint32_t tab_lookup(uint32_t word, uint32_t lane4x, uint32_t sel) {
  const uint32_t addr = __byte_perm(word, lane4x, sel);
  uint32_t r;
  asm("ld.shared.b32 %0, [%1];" : "=r"(r) : "r"(addr));
  return r;
}

// one 64-column scale group of one 16-row strip: 4 MMAs; returns hi+lo sums for rows g, g+8
__device__ __forceinline__ void group_mma(uint2 ca, uint2 cb, const uint32_t (&bq)[8], uint32_t lane4x, float& r_g,
                                          float& r_h) {
  // two independent accumulator chains (k-steps 0,2 and 1,3) halve the MMA dependency depth
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t a[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t wa = (j < 2) ? ca.x : ca.y;
    const uint32_t wb = (j < 2) ? cb.x : cb.y;
    const uint32_t k0 = 2 * (j & 1);
    const uint32_t s0 = 0x6504u | (k0 << 4), s1 = 0x6504u | ((k0 + 1) << 4);
    a[j][0] = tab_lookup(wa, lane4x, s0);  // row g,   pair 8q+2j
    a[j][1] = tab_lookup(wb, lane4x, s0);  // row g+8, pair 8q+2j
    a[j][2] = tab_lookup(wa, lane4x, s1);  // row g,   pair 8q+2j+1
    a[j][3] = tab_lookup(wb, lane4x, s1);  // row g+8, pair 8q+2j+1
  }
  mma_bf16_16816(d0, a[0], bq[0], bq[1], d0);
  mma_bf16_16816(d1, a[1], bq[2], bq[3], d1);
  mma_bf16_16816(d0, a[2], bq[4], bq[5], d0);
  mma_bf16_16816(d1, a[3], bq[6], bq[7], d1);
  r_g = (d0[0] + d1[0]) + (d0[1] + d1[1]);
  r_h = (d0[2] + d1[2]) + (d0[3] + d1[3]);
}

__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

struct StripInfo {
  int m0;     // matrix of the strip (the first of the pair in SwiGLU mode)
  int rbase;  // first row of the strip within that matrix
};

template <int NMAT>
__device__ __forceinline__ StripInfo strip_info(const HexmvParams& P, int s) {
  StripInfo si;
  if (NMAT == 2) {
    si.m0 = 0;
    si.rbase = s * 16;
  } else {
    int m = 0;
    while (m < P.job.n_mat - 1 && s >= P.strip_begin[m + 1]) ++m;
    si.m0 = m;
    si.rbase = (s - P.strip_begin[m]) * 16;
  }
  return si;
}

// Epilogue of a completed strip.  Lane j holds the finished value of row (j & 15) of
// matrix m0 + (j >> 4) (lanes >= 16 only carry data in pair mode).
template <int EPI>
__device__ void strip_epilogue(const HexmvParams& P, const StripInfo& si, float v, int lane) {
  const gsdlq_linear_job_t& J = P.job;
  const int r = lane & 15;
  const gsdlq_hexmat_t& M = J.mat[si.m0];
  const int row = si.rbase + r;
  const bool ok = row < M.rows;
  if constexpr (EPI == GSDLQ_EPI_STORE) {
    unsigned long long key = 0ull;
    if (lane < 16 && ok) {
      J.y[si.m0][row] = v;
      if (J.argmax_key) key = argmax_key(v, (uint32_t)(row + J.argmax_index_base));
    }
    if (J.argmax_key) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (lane == 0 && key) atomicMax(J.argmax_key, key);
    }
  } else if constexpr (EPI == GSDLQ_EPI_RESID) {
    if (lane < 16 && ok) J.y[0][row] = J.resid[row] + v;
  } else if constexpr (EPI == GSDLQ_EPI_SWIGLU) {
    const float u = __shfl_down_sync(0xffffffffu, v, 16);
    if (lane < 16 && ok) J.y[0][row] = (v / (1.0f + expf(-v))) * u;
  } else if constexpr (EPI == GSDLQ_EPI_ROPE_KV) {
    // rows (2i, 2i+1) of a head form one interleaved RoPE pair
    const float other = __shfl_xor_sync(0xffffffffu, v, 1);
    if (lane < 16 && ok) {
      const bool even = (r & 1) == 0;
      const float v0 = even ? v : other, v1 = even ? other : v;
      const int pos = *J.pos;
      const int hd = J.head_dim;
      const bool pos_ok = pos >= 0 && pos < J.max_seq;
      if (!pos_ok && lane == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
      if (si.m0 == 2) {  // V: stored unrotated
        if (J.y[2]) J.y[2][row] = v;
        if (pos_ok) J.v_cache[((size_t)J.layer * J.max_seq + pos) * M.rows + row] = f2h(v);
      } else {
        const int i = (row % hd) >> 1;
        const float2 cs = pos_ok ? reinterpret_cast<const float2*>(J.rope_cs)[(size_t)pos * (hd / 2) + i]
                                 : make_float2(1.f, 0.f);
        const float o = even ? __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y))
                             : __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
        if (si.m0 == 0) {
          J.y[0][row] = o;
        } else {
          if (J.y[1]) J.y[1][row] = o;
          if (pos_ok) J.k_cache[((size_t)J.layer * J.max_seq + pos) * M.rows + row] = f2h(o);
        }
      }
    }
  }
}

// Sum a completed strip's slots in slot order and run its epilogue (one warp).
template <int EPI, int NMAT>
__device__ void finish_strip(const HexmvParams& P, int s, int lane) {
  __threadfence();
  const int GU = P.GU;
  const int w_first = warp_of((long long)s * GU, P.T, P.W);
  const int w_last = warp_of((long long)s * GU + GU - 1, P.T, P.W);
  const int nseg = w_last - w_first + 1;
  constexpr int width = NMAT * 16;
  const float* base = P.part + (size_t)s * (P.max_seg + 1) * width;
  float v = 0.f;
  if (lane < width) {
    float* bw = const_cast<float*>(base);
    for (int k = 0; k < nseg; ++k) {
      v += ld_cg_f32(base + (size_t)k * width + lane);
      bw[(size_t)k * width + lane] = 0.f;
    }
    v += ld_cg_f32(base + (size_t)P.max_seg * width + lane);  // helper slot: kinks + low rank
    bw[(size_t)P.max_seg * width + lane] = 0.f;
  }
  // every consumed slot and the counter go back to zero: the whole workspace is zero between
  // launches, so launches of any geometry can share it
  if (lane == 0) P.cnt[s] = 0u;
  strip_epilogue<EPI>(P, strip_info<NMAT>(P, s), v, lane);
}

// Count `units` toward strip s after this warp's slot writes; the warp completing the
// strip (GU streaming units + 1 helper unit) finishes it.
template <int EPI, int NMAT>
__device__ __forceinline__ void arrive(const HexmvParams& P, int s, unsigned units, int lane, bool fence = true) {
  if (fence) __threadfence();  // every lane that wrote part of the slot orders its stores before the count
  __syncwarp();
  unsigned fin = 0;
  if (lane == 0) {
    const unsigned old = atomicAdd(&P.cnt[s], units);
    fin = (old + units == (unsigned)P.GU + 1u);
  }
  fin = __shfl_sync(0xffffffffu, fin, 0);
  if (fin) finish_strip<EPI, NMAT>(P, s, lane);
}

template <int EPI, int UG>
__global__ void __launch_bounds__(HX_THREADS, 1) hexmv_kernel(const __grid_constant__ HexmvParams P) {
  constexpr int NMAT = (EPI == GSDLQ_EPI_SWIGLU) ? 2 : 1;
  extern __shared__ __align__(1024) uint8_t smem[];
  const gsdlq_linear_job_t& J = P.job;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gl = lane >> 2, q = lane & 3;
  const int C = P.cols, G = P.G, NP = P.NP;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  if (sbase > (uint32_t)HX_BASE_MAX || (sbase & 15u)) {  // the layout's assumption on the reserved bytes
    if (tid == 0) raise_flag(GSDLQ_FLAG_UNSUPPORTED);
    return;
  }
  const uint32_t tab_off = HX_TAB_ABS - sbase;
  uint8_t* tab = smem + tab_off;
  float* xf = reinterpret_cast<float*>(smem + tab_off + HX_TAB_ABS);
  const HxLayout LY = hx_layout(P.ovf_bytes, P.sc_strips, NMAT, G);
  uint32_t* s_sc = reinterpret_cast<uint32_t*>(smem + LY.sc_off);
  float* misc = reinterpret_cast<float*>(smem + LY.misc_off);  // [0] 1/rms, [1..16] reduction

  // ---- 1. independent prologue: decode table, this CTA's scale window, first code prefetches
  build_decode_table(tab, P);
  const int w_cta0 = blockIdx.x * HX_STREAM;
  const long long cta_u0 = it_begin(min(w_cta0, P.W), P.T, P.W);
  const long long cta_u1 = it_begin(min(w_cta0 + HX_STREAM, P.W), P.T, P.W);
  const int sc_first = (int)(cta_u0 / P.GU);
  const int sc_n = (cta_u1 > cta_u0) ? (int)((cta_u1 - 1) / P.GU) - sc_first + 1 : 0;
  const int scw_n = hx_sc_words(G);
  {
    // asynchronous 4-byte copies of whole rows (2-byte loads when G is odd and rows are not
    // 4-byte aligned)
    const int n_rows = sc_n * NMAT * 16;
    for (int rid = warp; rid < n_rows; rid += HX_WARPS) {
      const int ls = rid / (NMAT * 16), rem = rid - ls * NMAT * 16;
      const int mm = rem >> 4, rr = rem & 15;
      const StripInfo si = strip_info<NMAT>(P, sc_first + ls);
      const gsdlq_hexmat_t& M = J.mat[si.m0 + mm];
      const int row = min(si.rbase + rr, M.rows - 1);
      const uint16_t* src = M.scales + (size_t)row * G;
      uint32_t* dst = s_sc + (size_t)rid * scw_n;
      if ((G & 1) == 0) {
        for (int wi = lane; wi < G / 2; wi += 32) cp_async_4(dst + wi, src + 2 * wi);
      } else {
        for (int gg = lane; gg < G; gg += 32) reinterpret_cast<uint16_t*>(dst)[gg] = __ldg(src + gg);
      }
    }
    cp_async_commit();
  }
  const int w = w_cta0 + warp;
  const bool streamer = warp < HX_STREAM && w < P.W;
  const long long u0 = streamer ? it_begin(w, P.T, P.W) : 0;
  const long long u1 = streamer ? it_begin(w + 1, P.T, P.W) : 0;
  const int GU = P.GU;
  uint2 pf[NMAT][UG][2];  // codes of the next unit: [matrix][group][row g / row g+8]
  // prefetch cursor: unit (strip pf_s, unit-in-strip pf_u) and this lane's code pointers
  int pf_s = (int)(u0 / GU), pf_u = (int)(u0 - (long long)pf_s * GU);
  const uint8_t* pfa[NMAT];
  const uint8_t* pfb[NMAT];
  auto seek = [&]() {
    const StripInfo si = strip_info<NMAT>(P, pf_s);
#pragma unroll
    for (int mm = 0; mm < NMAT; ++mm) {
      const gsdlq_hexmat_t& M = J.mat[si.m0 + mm];
      const int ra = min(si.rbase + gl, M.rows - 1), rb = min(si.rbase + gl + 8, M.rows - 1);
      pfa[mm] = M.codes + (size_t)ra * NP + pf_u * (UG * 32) + q * 8;
      pfb[mm] = M.codes + (size_t)rb * NP + pf_u * (UG * 32) + q * 8;
    }
  };
  auto issue = [&]() {
#pragma unroll
    for (int mm = 0; mm < NMAT; ++mm) {
#pragma unroll
      for (int k = 0; k < UG; ++k) {
        pf[mm][k][0] = ldg_stream_u2(pfa[mm] + 32 * k);
        pf[mm][k][1] = ldg_stream_u2(pfb[mm] + 32 * k);
      }
      pfa[mm] += UG * 32;
      pfb[mm] += UG * 32;
    }
    if (++pf_u == GU) {
      pf_u = 0;
      ++pf_s;
      seek();
    }
  };
  if (streamer && u1 > u0) {
    seek();
    issue();
  }

  // ---- 2. wait for the producer of x, then stage the input (fp32 and bf16 splits) ----------
  pdl_wait();
  int tok = 0;
  if (J.input_mode == GSDLQ_IN_EMBED) {
    tok = *J.token;
    if (tok < 0 || tok >= J.vocab) {
      if (tid == 0) raise_flag(GSDLQ_FLAG_BAD_TOKEN);
      tok = 0;
    }
  }
  float inv = 1.f;
  if (J.input_mode != GSDLQ_IN_PLAIN) {
    float ss = 0.f;
    for (int c = tid; c < C; c += HX_THREADS) {
      const float v = (J.input_mode == GSDLQ_IN_EMBED) ? h2f(__ldg(J.embed + (size_t)tok * C + c)) : __ldg(J.x + c);
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) misc[1 + warp] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int k = 0; k < HX_WARPS; ++k) t += misc[1 + k];
      misc[0] = 1.0f / sqrtf(t / (float)C + J.eps);  // gsd_lq_cpu_engine.c:78
    }
    __syncthreads();
    inv = misc[0];
  }
  // loads of a batch are issued before any shared store, so they overlap (the generic input
  // pointers could otherwise be assumed to alias shared memory and serialise)
  constexpr int XB = 8;
  for (int p0 = tid; p0 < NP; p0 += XB * HX_THREADS) {
    float2 xv[XB], wv[XB];
#pragma unroll
    for (int k = 0; k < XB; ++k) {
      const int p = p0 + k * HX_THREADS;
      if (p < NP) {
        if (J.input_mode == GSDLQ_IN_EMBED) {
          const uint32_t raw = __ldg(reinterpret_cast<const unsigned int*>(J.embed + (size_t)tok * C) + p);
          xv[k] = make_float2(h2f(raw & 0xffffu), h2f(raw >> 16));
        } else {
          xv[k] = __ldg(reinterpret_cast<const float2*>(J.x) + p);
        }
        wv[k] = (J.input_mode != GSDLQ_IN_PLAIN) ? __ldg(reinterpret_cast<const float2*>(J.norm_w) + p)
                                                 : make_float2(1.f, 1.f);
      }
    }
#pragma unroll
    for (int k = 0; k < XB; ++k) {
      const int p = p0 + k * HX_THREADS;
      if (p < NP) {
        float x0 = xv[k].x, x1 = xv[k].y;
        if (J.input_mode == GSDLQ_IN_EMBED && blockIdx.x == 0 && J.x_out)
          reinterpret_cast<float2*>(J.x_out)[p] = make_float2(x0, x1);
        if (J.input_mode != GSDLQ_IN_PLAIN) {
          x0 = __fmul_rn(__fmul_rn(x0, inv), wv[k].x);
          x1 = __fmul_rn(__fmul_rn(x1, inv), wv[k].y);
        }
        reinterpret_cast<float2*>(xf)[p] = make_float2(x0, x1);
        const float b = fmaf(0.8660254037844386f, x1, 0.5f * x0);
        uint32_t h, l;
        split_bf16x2(x0, b, h, l);
        // pair i of group g: hi word at i*4 of chunk 2g; lo word in chunk 2g+1 with the two
        // 16-byte halves of each 32-byte lane segment swapped (see the B-fragment loads)
        const int g = p >> 5, i = p & 31;
        const int ilo = (i & ~7) | ((i + 4) & 7);
        *reinterpret_cast<uint32_t*>(smem + xs_chunk(2 * g, tab_off) + 4 * i) = h;
        *reinterpret_cast<uint32_t*>(smem + xs_chunk(2 * g + 1, tab_off) + 4 * ilo) = l;
      }
    }
  }
  if (tid == 0) reinterpret_cast<uint32_t*>(misc)[32] = 0x0100u;  // table address bits 16..23, read after the barrier
  cp_async_wait_all();  // the staged scale window
  __syncthreads();

  if (warp >= HX_STREAM) {
    // ---- helper warps: low-rank projections, then per-strip kink + low-rank slots --------
    unsigned* ctl = P.ctl;
    while (true) {
      unsigned t = 0;
      if (lane == 0) t = atomicAdd(&ctl[CTL_TK_TICKET], 1u);
      t = __shfl_sync(0xffffffffu, t, 0);
      if ((int)t >= P.n_lr_jobs) break;
      int m = 0, j = (int)t;
      while (m < J.n_mat - 1 && j >= J.mat[m].k_dim) j -= J.mat[m].k_dim, ++m;
      const gsdlq_hexmat_t& M = J.mat[m];
      const uint4* vt = reinterpret_cast<const uint4*>(M.Vt + (size_t)j * C);
      float acc = 0.f;
      for (int c8 = lane; c8 < C / 8; c8 += 4 * 32) {
        uint4 raw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) raw[u] = (c8 + 32 * u < C / 8) ? __ldg(vt + c8 + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (c8 + 32 * u < C / 8) {
            const float4* xp = reinterpret_cast<const float4*>(xf + 8 * (c8 + 32 * u));
            const float4 a = xp[0], b = xp[1];
            acc += a.x * h2f(raw[u].x & 0xffffu) + a.y * h2f(raw[u].x >> 16) + a.z * h2f(raw[u].y & 0xffffu) +
                   a.w * h2f(raw[u].y >> 16) + b.x * h2f(raw[u].z & 0xffffu) + b.y * h2f(raw[u].z >> 16) +
                   b.z * h2f(raw[u].w & 0xffffu) + b.w * h2f(raw[u].w >> 16);
          }
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) {
        reinterpret_cast<volatile float*>(ctl)[CTL_TMPK + m * 16 + j] = acc * M.S[j];
        __threadfence();
        atomicAdd(&ctl[CTL_TK_DONE], 1u);
      }
    }
    if (P.n_lr_jobs > 0) {
      if (lane == 0) wait_counter_geq(&ctl[CTL_TK_DONE], (unsigned)P.n_lr_jobs, 1000000000ull);  // 1 s bound
      __syncwarp();
      __threadfence();
    }
    constexpr int width = NMAT * 16;
    while (true) {
      unsigned s = 0;
      if (lane == 0) s = atomicAdd(&ctl[CTL_KINK_TICKET], 1u);
      s = __shfl_sync(0xffffffffu, s, 0);
      if ((int)s >= P.n_strips) break;
      const StripInfo si = strip_info<NMAT>(P, (int)s);
      const int r = lane & 15, hi = lane >> 4;
      const int mm = (NMAT == 2) ? hi : 0;
      const gsdlq_hexmat_t& M = J.mat[si.m0 + mm];
      const int row = si.rbase + r;
      float v = 0.f;
      if (row < M.rows) {
        // low-rank term first: its U loads do not depend on row_ptr
        if (M.k_dim > 0 && (NMAT == 2 || hi == 0)) {
          const uint16_t* ur = M.U + (size_t)row * M.k_dim;
          uint16_t uv[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) uv[jj] = jj < M.k_dim ? __ldg(ur + jj) : (uint16_t)0;
          const float* tk = P.tmp_k_ext ? P.tmp_k_ext : reinterpret_cast<const float*>(ctl) + CTL_TMPK + (si.m0 + mm) * 16;
#pragma unroll
          for (int jj = 0; jj < 16; ++jj)
            if (jj < M.k_dim) v += h2f(uv[jj]) * __ldcg(tk + jj);
        }
        const uint32_t e0 = __ldg(M.row_ptr + row), e1 = __ldg(M.row_ptr + row + 1);
        constexpr int step = (NMAT == 2) ? 1 : 2;
        // kinks in batches of 16: the batch's loads are issued together
        for (uint32_t e = e0 + (NMAT == 2 ? 0 : hi); e < e1; e += 16 * step) {
          int col[16];
          float dl[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const uint32_t eu = e + u * step;
            col[u] = eu < e1 ? (int)__ldg(M.kink_cols + eu) : 0;
            dl[u] = eu < e1 ? __ldg(M.kink_deltas + eu) : 0.f;
          }
          bool bad = false;
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const bool ok = col[u] < C;
            v += ok ? dl[u] * xf[ok ? col[u] : 0] : 0.f;
            bad |= !ok;
          }
          if (bad) raise_flag(GSDLQ_FLAG_BAD_KINK);
        }
      }
      if (NMAT == 1) v += __shfl_xor_sync(0xffffffffu, v, 16);
      float* slot = P.part + ((size_t)s * (P.max_seg + 1) + P.max_seg) * width;
      if (lane < width) slot[lane] = v;
      arrive<EPI, NMAT>(P, (int)s, 1u, lane);
    }
  } else if (streamer) {
    // ---- streaming warps --------------------------------------------------------------
    const uint32_t lane4x = (uint32_t)lane * 4u | reinterpret_cast<const volatile uint32_t*>(misc)[32];
    // B fragments: lane (gl, q) supplies column n = gl of B.  Column 0 is the hi split, column 1
    // the lo split; the lo chunk stores each lane segment's halves swapped, so the 8 lanes of
    // columns 0-1 touch 32 distinct banks per 16-byte load and all receive pairs 0-3 first.
    // Columns 2-7 only feed D columns 2-7, which are never read, so lanes gl >= 2 simply load the
    // same addresses as lanes gl & 1 (a broadcast: no extra wavefronts, no divergent branch).
    const int gb = gl & 1;
    const uint32_t boff0 = (uint32_t)(q * 32 + 16 * gb), boff1 = (uint32_t)(q * 32 + 16 * (1 - gb));
    int cur_s = (int)(u0 / GU), cur_u = (int)(u0 - (long long)cur_s * GU);
    int seg_s = cur_s;
    float acc[NMAT][2];
#pragma unroll
    for (int mm = 0; mm < NMAT; ++mm) acc[mm][0] = acc[mm][1] = 0.f;
    auto emit = [&](int s) {
      const int seg = w - warp_of((long long)s * GU, P.T, P.W);
      constexpr int width = NMAT * 16;
      float* slot = P.part + ((size_t)s * (P.max_seg + 1) + seg) * width;
      if (q == 0) {
#pragma unroll
        for (int mm = 0; mm < NMAT; ++mm) {
          slot[mm * 16 + gl] = acc[mm][0];
          slot[mm * 16 + gl + 8] = acc[mm][1];
        }
      }
    };
    for (long long u = u0; u < u1; ++u) {
      if (cur_s != seg_s) {
        emit(seg_s);
        seg_s = cur_s;
#pragma unroll
        for (int mm = 0; mm < NMAT; ++mm) acc[mm][0] = acc[mm][1] = 0.f;
      }
      uint2 cur[NMAT][UG][2];
#pragma unroll
      for (int mm = 0; mm < NMAT; ++mm)
#pragma unroll
        for (int k = 0; k < UG; ++k) {
          cur[mm][k][0] = pf[mm][k][0];
          cur[mm][k][1] = pf[mm][k][1];
        }
      if (u + 1 < u1) issue();
      // this lane's staged scale rows (gl and gl + 8) of the unit's strip
      const uint16_t* sra = reinterpret_cast<const uint16_t*>(s_sc + ((size_t)((cur_s - sc_first) * NMAT) * 16 + gl) * scw_n);
#pragma unroll
      for (int k = 0; k < UG; ++k) {
        const int g = cur_u * UG + k;
        const uint8_t* src = smem + xs_chunk(2 * g + gb, tab_off);
        const uint4 v0 = *reinterpret_cast<const uint4*>(src + boff0);
        const uint4 v1 = *reinterpret_cast<const uint4*>(src + boff1);
        const uint32_t bq[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int mm = 0; mm < NMAT; ++mm) {
          const uint16_t* sr = sra + (size_t)mm * 16 * scw_n * 2;
          const float sa = h2f(sr[g]), sb = h2f(sr[8 * scw_n * 2 + g]);
          float rg, rh;
          group_mma(cur[mm][k][0], cur[mm][k][1], bq, lane4x, rg, rh);
          acc[mm][0] = fmaf(sa, rg, acc[mm][0]);
          acc[mm][1] = fmaf(sb, rh, acc[mm][1]);
        }
      }
      if (++cur_u == GU) {
        cur_u = 0;
        ++cur_s;
      }
    }
    if (u1 > u0) {
      emit(seg_s);
      // the counts are deferred to the end of the range: a fence mid-range would wait for the code
      // prefetches in flight.  One fence covers all of this warp's slot stores, then one count per
      // strip the range touched.
      __threadfence();
      const int s_a = (int)(u0 / GU), s_b = (int)((u1 - 1) / GU);
      for (int s = s_a; s <= s_b; ++s) {
        const long long a = max(u0, (long long)s * GU), b = min(u1, (long long)s * GU + GU);
        arrive<EPI, NMAT>(P, s, (unsigned)(b - a), lane, false);
      }
    }
  }

  pdl_launch_dependents();
  // ---- the last CTA leaves the control words at zero for the next launch ---------------
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&P.ctl[CTL_DONE], 1u) == gridDim.x - 1) {
      for (int i = 0; i < CTL_WORDS; ++i) P.ctl[i] = 0u;
      __threadfence();
    }
  }
}

// ---- host side ------------------------------------------------------------------------
static int hexmv_validate_mat(const gsdlq_hexmat_t& M, int cols, bool own_lowrank) {
  if (!M.codes || !M.scales || !M.row_ptr) return GSDLQ_ERR_INVALID;
  // codes are read 8 bytes at a time from row starts (cols/2 is a multiple of 32)
  if (reinterpret_cast<uintptr_t>(M.codes) & 7u) return GSDLQ_ERR_INVALID;
  if (M.rows <= 0 || M.cols != cols || cols <= 0 || cols % 64 != 0) return GSDLQ_ERR_INVALID;
  if (M.k_dim < 0 || M.k_dim > 16) return GSDLQ_ERR_INVALID;
  if (M.k_dim > 0 && !M.U) return GSDLQ_ERR_INVALID;
  if (own_lowrank && M.k_dim > 0 && (!M.S || !M.Vt)) return GSDLQ_ERR_INVALID;
  if (own_lowrank && M.k_dim > 0 && (reinterpret_cast<uintptr_t>(M.Vt) & 15u)) return GSDLQ_ERR_INVALID;  // 16-byte loads
  if (M.radius != 6 && M.radius != 8) return GSDLQ_ERR_INVALID;
  return GSDLQ_OK;
}

// Geometry of a launch (everything but the workspace pointers).
static int hexmv_plan(HexmvParams& P) {
  const gsdlq_linear_job_t& J = P.job;
  if (J.n_mat < 1 || J.n_mat > 3) return GSDLQ_ERR_INVALID;
  const int C = J.mat[0].cols;
  for (int m = 0; m < J.n_mat; ++m) {
    const int st = hexmv_validate_mat(J.mat[m], C, P.tmp_k_ext == nullptr);
    if (st != GSDLQ_OK) return st;
    if (J.mat[m].radius != J.mat[0].radius) return GSDLQ_ERR_INVALID;
  }
  P.cols = C;
  P.G = C / 64;
  P.NP = C / 2;
  if (C > 65535) return GSDLQ_ERR_UNSUPPORTED;  // u16 kink columns
  P.nmat = (J.epilogue == GSDLQ_EPI_SWIGLU) ? 2 : 1;
  if (P.nmat == 2) {
    if (J.n_mat != 2) return GSDLQ_ERR_INVALID;
    P.n_strips = (J.mat[0].rows + 15) / 16;
  } else {
    P.strip_begin[0] = 0;
    for (int m = 0; m < J.n_mat; ++m) P.strip_begin[m + 1] = P.strip_begin[m] + (J.mat[m].rows + 15) / 16;
    P.n_strips = P.strip_begin[J.n_mat];
  }
  // work unit: UG consecutive groups of one strip (4, or 2 in pair mode, when G allows)
  const int ug_max = (P.nmat == 2) ? 2 : 4;
  P.UG = (P.G % ug_max == 0) ? ug_max : ((P.G % 2 == 0) ? 2 : 1);
  P.GU = P.G / P.UG;
  P.T = (long long)P.n_strips * P.GU;
  const int max_w = num_sms() * HX_STREAM;
  P.W = (int)std::min<long long>(max_w, P.T);
  const long long lmin = P.T / P.W;
  P.max_seg = (int)((P.GU - 1 + lmin - 1) / lmin) + 1;
  int lr = 0;
  for (int m = 0; m < J.n_mat; ++m) lr += J.mat[m].k_dim;
  P.n_lr_jobs = P.tmp_k_ext ? 0 : lr;
  // staged-scale window: the most strips one CTA's 14 warps touch
  const int grid = (P.W + HX_STREAM - 1) / HX_STREAM;
  int sc = 1;
  for (int c = 0; c < grid; ++c) {
    const long long a = it_begin(std::min(c * HX_STREAM, P.W), P.T, P.W);
    const long long b = it_begin(std::min((c + 1) * HX_STREAM, P.W), P.T, P.W);
    if (b > a) sc = std::max(sc, (int)((b - 1) / P.GU - a / P.GU + 1));
  }
  P.sc_strips = sc;
  P.ovf_bytes = std::max(0, 2 * P.G - 256) * 128;
  return GSDLQ_OK;
}

template <int EPI, int UG>
static int hexmv_launch_t(const HexmvParams& P, cudaStream_t s) {
  const HxLayout LY = hx_layout(P.ovf_bytes, P.sc_strips, P.nmat, P.G);
  const int dyn = hx_dyn_smem(P.cols);
  if (LY.low_end > (int)HX_TAB_ABS - HX_BASE_MAX || dyn > 227 * 1024) return GSDLQ_ERR_UNSUPPORTED;
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(hexmv_kernel<EPI, UG>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return record_cuda_error(e);
    configured[dev] = true;
  }
  const int grid = (P.W + HX_STREAM - 1) / HX_STREAM;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(HX_THREADS);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, hexmv_kernel<EPI, UG>, P);
  if (e != cudaSuccess) return record_cuda_error(e);
  return GSDLQ_OK;
}

static int hexmv_check_io(const HexmvParams& P) {
  const gsdlq_linear_job_t& J = P.job;
  if (J.input_mode < 0 || J.input_mode > 2) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_PLAIN && !J.x) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_RMSNORM && (!J.x || !J.norm_w)) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_EMBED && (!J.embed || !J.token || !J.norm_w || J.vocab <= 0)) return GSDLQ_ERR_INVALID;
  if (J.input_mode != GSDLQ_IN_EMBED && (reinterpret_cast<uintptr_t>(J.x) & 7u)) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_EMBED && (reinterpret_cast<uintptr_t>(J.embed) & 3u)) return GSDLQ_ERR_INVALID;
  switch (J.epilogue) {
    case GSDLQ_EPI_STORE:
      if (J.n_mat != 1 && J.argmax_key) return GSDLQ_ERR_INVALID;
      for (int m = 0; m < J.n_mat; ++m)
        if (!J.y[m]) return GSDLQ_ERR_INVALID;
      return GSDLQ_OK;
    case GSDLQ_EPI_RESID:
      return (J.n_mat != 1 || !J.y[0] || !J.resid) ? GSDLQ_ERR_INVALID : GSDLQ_OK;
    case GSDLQ_EPI_SWIGLU:
      return (J.n_mat != 2 || !J.y[0] || J.mat[0].rows != J.mat[1].rows) ? GSDLQ_ERR_INVALID : GSDLQ_OK;
    case GSDLQ_EPI_ROPE_KV:
      if (J.n_mat != 3 || !J.y[0] || !J.k_cache || !J.v_cache || !J.pos || !J.rope_cs) return GSDLQ_ERR_INVALID;
      if (J.interleaved != 1 || J.head_dim <= 0 || J.head_dim % 16 != 0 || J.max_seq <= 0) return GSDLQ_ERR_UNSUPPORTED;
      if (J.mat[1].rows != J.mat[2].rows || J.mat[0].rows % J.head_dim || J.mat[1].rows % J.head_dim)
        return GSDLQ_ERR_INVALID;
      return GSDLQ_OK;
    default:
      return GSDLQ_ERR_INVALID;
  }
}

template <int EPI>
static int hexmv_dispatch_ug(const HexmvParams& P, cudaStream_t s) {
  if constexpr (EPI != GSDLQ_EPI_SWIGLU) {  // pair mode never uses 4-group units
    if (P.UG == 4) return hexmv_launch_t<EPI, 4>(P, s);
  }
  if (P.UG == 2) return hexmv_launch_t<EPI, 2>(P, s);
  return hexmv_launch_t<EPI, 1>(P, s);
}

static int hexmv_dispatch(const HexmvParams& P, cudaStream_t s) {
  switch (P.job.epilogue) {
    case GSDLQ_EPI_STORE: return hexmv_dispatch_ug<GSDLQ_EPI_STORE>(P, s);
    case GSDLQ_EPI_RESID: return hexmv_dispatch_ug<GSDLQ_EPI_RESID>(P, s);
    case GSDLQ_EPI_SWIGLU: return hexmv_dispatch_ug<GSDLQ_EPI_SWIGLU>(P, s);
    default: return hexmv_dispatch_ug<GSDLQ_EPI_ROPE_KV>(P, s);
  }
}

int hexmv_launch(HexmvParams& P, void* workspace, size_t ws_bytes, cudaStream_t s) {
  int st = hexmv_plan(P);
  if (st != GSDLQ_OK) return st;
  st = hexmv_check_io(P);
  if (st != GSDLQ_OK) return st;
  const size_t need = hexmv_ws_bytes_for(P.n_strips, P.max_seg, P.nmat);
  if (!workspace || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u)) return GSDLQ_ERR_INVALID;
  P.ctl = static_cast<unsigned*>(workspace);
  P.cnt = P.ctl + CTL_WORDS;
  const uintptr_t pb = reinterpret_cast<uintptr_t>(P.cnt + P.n_strips);
  P.part = reinterpret_cast<float*>((pb + 15) & ~uintptr_t(15));
  return hexmv_dispatch(P, s);
}

size_t hexmv_ws_bytes(HexmvParams& P) {
  if (hexmv_plan(P) != GSDLQ_OK) return 0;
  return hexmv_ws_bytes_for(P.n_strips, P.max_seg, P.nmat);
}

// Workspace of the drop-in gsdlq_hex2d_matvec, whose signature carries none: one buffer
// per device, allocated on first use, grown on demand, zero-initialised.
struct DropinWs {
  void* p = nullptr;
  size_t bytes = 0;
};
static DropinWs g_mv_ws[64];

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_linear_ws_size(const gsdlq_linear_job_t* job, size_t* bytes) {
  if (!job || !bytes) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  P.job = *job;
  const size_t b = hexmv_ws_bytes(P);
  if (b == 0) return GSDLQ_ERR_INVALID;
  *bytes = b;
  return GSDLQ_OK;
}

extern "C" int gsdlq_linear(const gsdlq_linear_job_t* job, void* workspace, size_t workspace_bytes,
                            gsdlq_stream_t stream) {
  if (!job) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  P.job = *job;
  return hexmv_launch(P, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
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
  M.row_ptr = kink_row_ptr;
  M.kink_cols = kink_cols;
  M.kink_deltas = kink_deltas;
  M.rows = rows;
  M.cols = cols;
  M.k_dim = k_dim;
  M.radius = 8;  // unused when xy_table is given
  // the drop-in signature carries no S/Vt: the low-rank term comes from the caller's tmp_k
  M.S = nullptr;
  M.Vt = nullptr;
  J.input_mode = GSDLQ_IN_PLAIN;
  J.x = x;
  J.epilogue = GSDLQ_EPI_STORE;
  J.y[0] = y;
  P.xy_table = xy_table;
  P.n_pts = n_pts;
  P.tmp_k_ext = k_dim > 0 ? tmp_k : nullptr;
  const size_t need = hexmv_ws_bytes(P);
  if (need == 0) return GSDLQ_ERR_INVALID;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e);
  if (dev < 0 || dev >= 64) return GSDLQ_ERR_UNSUPPORTED;
  DropinWs& ws = g_mv_ws[dev];
  if (ws.bytes < need) {
    if (ws.p) cudaFree(ws.p);
    ws.p = nullptr;
    ws.bytes = 0;
    e = cudaMalloc(&ws.p, need);
    if (e != cudaSuccess) return record_cuda_error(e);
    e = cudaMemset(ws.p, 0, need);
    if (e != cudaSuccess) return record_cuda_error(e);
    ws.bytes = need;
  }
  return hexmv_launch(P, ws.p, ws.bytes, static_cast<cudaStream_t>(stream));
}

// hexmv_dev.cuh -- device code of the fused GSD-LQ packed linear for batch-1 decode on sm_100a.
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
// mantissa bits together).  Warp-level mma.sync m16n8k16 (bf16 in, fp32
// accumulate) does the multiply-adds; the kernel is HBM-bound on the code
// stream (0.53 B/weight).
//
// Code stream.  A work unit is 16 rows x 256 code bytes (512 columns, 8 scale
// groups) of one matrix.  Lane (g, q) of a warp loads 16 contiguous bytes of rows
// g and g+8 at byte 64*s + 16*q of the unit (segment s = 0..3), so every load
// instruction reads 64 contiguous bytes per row and a unit reads 256 contiguous
// bytes per row -- the shape that streams HBM at full rate.  The unit's 8 fp16
// scales per row are one 16-byte load.  The next unit's loads are in flight
// while the current one is computed (segment by segment, in registers).
//
// Decode.  A code byte becomes its bf16x2 (r0, r1) through one byte-permute
// (PRMT: code -> bits 8..15, lane*4 -> bits 0..7) and one 32-bit shared load
// from a 256-entry table replicated once per lane in the lane's own bank
// (entry c of lane l at byte c*256 + l*4), so the 32 lookups of a warp never
// conflict.  The other half of every 256-byte table row holds staged
// activation splits.
//
// MMA shape.  Within a 64-byte segment, lanes q = 0,1 hold scale group A and
// lanes q = 2,3 hold group B.  One m16n8k16 per pair of k-steps takes A = decoded
// codes (16 rows x 8 code pairs, two from each lane) and a block-diagonal B:
// column 0/1 = hi/lo splits of group A's activations (zero on group B's k rows),
// column 2/3 = hi/lo of group B (zero on group A's k rows), columns 4-7 zero.
// Lane q = 0 then holds group A's dot products for rows g, g+8 and lane q = 1
// group B's, so each applies its own group's scale.
//
// Work split: persistent stream-K with a CTA-local reduction.  One CTA per SM:
// 14 streaming warps and 2 helper warps.  The (strip, matrix, unit) iterations
// of the launch are dealt to the CTAs as equal contiguous ranges and, inside a
// CTA, to the streaming warps in proportion to their issue share.  Every
// contribution to a 16-row strip is added in 2^-32 fixed point (64-bit integer
// sums, so the result does not depend on the order of the additions) into a
// shared-memory accumulator of the CTA.  The helper warps add the kink sums
// and the low-rank term of the strips whose first unit lies in their CTA: the
// low-rank projection tmp_k = S * (Vt . x) is computed once per launch in
// column slices by all helpers of the grid, or forwarded by the kernel that
// produced x.  After one CTA barrier a strip inside the CTA's range is
// finished from shared memory; for a strip shared with other CTAs every sharer
// adds its part, plus a count unit, to one global word per row with a returning
// atomic, and the CTA whose addition completes the count finishes the strip and
// leaves the words at zero.  An RMSNorm input is staged as w * x and the finished
// values are multiplied by 1/rms.
//
// Launch order (programmatic dependent launch): the next launch is released at
// once; decode table, the first unit's code and scale loads and L2 prefetches
// of the helpers' Vt slices are issued BEFORE griddepcontrol.wait, so they
// overlap the previous kernel; the input x is read only after it.
#pragma once
#include <cuda.h>  // CUtensorMap

#include <algorithm>
#include <cstdio>

#include "comm.cuh"
#include "common.cuh"

namespace gsdlq {

constexpr int HX_WARPS = 16;
constexpr int HX_STREAM = 14;
constexpr int HX_HELP = HX_WARPS - HX_STREAM;
constexpr int HX_THREADS = HX_WARPS * kWarp;
constexpr int HX_UB = 256;  // code bytes of one row in a work unit (8 scale groups, 512 columns)

// control words at the start of the workspace
constexpr int CTL_LR_DONE = 0;  // helper warps that have added their low-rank slice
constexpr int CTL_DONE = 1;     // CTAs finished
constexpr int CTL_TMPK = 16;    // 48 x u64 fixed-point low-rank accumulators (words 16..111)
constexpr int CTL_WORDS = 128;
constexpr float LR_FIX = 4294967296.f;  // 2^32: fixed-point scale of the low-rank partials
constexpr float LR_MAX = 4194304.f;     // 2^22: largest partial magnitude (keeps 296 partials in 63 bits)

struct HexmvParams {
  gsdlq_linear_job_t job;
  const float* xy_table;   // drop-in path: decode table derived from this float table
  const float* tmp_k_ext;  // drop-in path: caller-computed tmp_k for mat[0]
  int n_pts;
  int cols, G, NP;
  int n_strips, nmat;      // nmat: matrices per strip (2 in SwiGLU pair mode)
  int strip_begin[4];      // prefix of strips per matrix (non-pair modes)
  int GU;                  // units per row: ceil(G / 8)
  int UPS;                 // units per strip: nmat * GU
  long long T;             // units in the launch: n_strips * UPS
  int n_cta;               // CTAs that carry units (the launch may have more)
  int n_local;             // strips one CTA's unit range can touch (rows of its accumulator)
  int lacc_off;            // its accumulator in shared memory, bytes after the decode table
  int n_lr;                // low-rank rows projected in the kernel (0 with tmp_k_ext)
  int lr_off[4];           // prefix of k_dim over the matrices
  int lr_chunks;           // 8-column chunks of every Vt row per helper warp
  int ovf_bytes;           // activation-split overflow region
  int ukink;               // every matrix has per-unit kink lists: the streaming warps apply them
  int pf_ahead;            // FULL streams: each warp prefetches into L2 the unit this many units past the
                           // one it is loading, within the same row block (0: none)
  unsigned* ctl;
  unsigned* cnt;                // [n_strips] reserved (zero; the shared-strip words count their own contributions)
  unsigned long long* gacc;     // [n_strips][nmat * 16] fixed-point sums of those strips
  // Inside the persistent decode kernel (null in a stand-alone launch): the input is ready once
  // *dep >= dep_target; every finished strip and every CTA of the launch add 1 to *done;
  // *abort is set when a bounded wait gives up, after which every later wait returns at once.
  const unsigned* dep;
  unsigned dep_target;
  unsigned* done;
  unsigned* abort;
  // tensor parallelism (stand-alone RESID launches): the exchange the epilogue sums the ranks' strips through
  CommDesc ex;
  int ex_on;
};

// The fields of a fused linear that differ between the layers of a model: the matrices' data,
// the RMSNorm weight, the layer index and the launch's scratch.  A stand-alone launch reads them
// from its own parameters (HxPtrs); the persistent decode kernel from the current layer's record,
// so that one shape record per phase kind serves every layer.  Shape fields (rows, k_dim, radius,
// strides, partition) always come from the HexmvParams itself.
// TMA descriptors of a stand-alone launch's matrices (codes: 64-byte x 16-row boxes of the
// [rows][cols/2] byte array; scales: 8 x 16 boxes of the [rows][cols/64] fp16 array).
struct HxMaps {
  CUtensorMap codes[3];
  CUtensorMap scales[3];
};

struct HxPtrs {
  const HexmvParams& P;
  const HxMaps& T;
  __device__ __forceinline__ const CUtensorMap* tmap_codes(int m) const { return &T.codes[m]; }
  __device__ __forceinline__ const CUtensorMap* tmap_scales(int m) const { return &T.scales[m]; }
  __device__ __forceinline__ const gsdlq_hexmat_t& mat(int m) const { return P.job.mat[m]; }
  __device__ __forceinline__ const float* norm_w() const { return P.job.norm_w; }
  __device__ __forceinline__ int layer() const { return P.job.layer; }
  __device__ __forceinline__ unsigned* ctl() const { return P.ctl; }
  __device__ __forceinline__ unsigned* cnt() const { return P.cnt; }
  __device__ __forceinline__ unsigned long long* gacc() const { return P.gacc; }
  __device__ __forceinline__ const unsigned* dep() const { return P.dep; }
  __device__ __forceinline__ unsigned dep_target() const { return P.dep_target; }
  __device__ __forceinline__ unsigned* done() const { return P.done; }
  __device__ __forceinline__ unsigned* abort() const { return P.abort; }
  __device__ __forceinline__ int input_mode() const { return P.job.input_mode; }
};

// ---- partition (identical on host and device) ---------------------------------------
// The (strip, matrix, unit) iterations are dealt to the CTAs as equal contiguous ranges, and a
// CTA's range to its 14 streaming warps as contiguous ranges weighted by scheduler: warps are
// spread over the SM's four schedulers by warp index mod 4, so schedulers 0 and 1 run four
// streaming warps and schedulers 2 and 3 run three plus one helper warp.  A warp on the second pair
// streams faster (its scheduler is shared by fewer streaming warps), but not 4/3 faster: a phase
// trace of the gate/up launch measured a per-unit rate ratio of 1.14, so the units are dealt in
// proportion 7 : 8.  lp(l) = sum of the weights of local warps 0 .. l-1.
__host__ __device__ __forceinline__ int hx_lp(int l) {
  const int r = l % 4;
  return 30 * (l / 4) + 7 * (r < 2 ? r : 2) + 8 * (r > 2 ? r - 2 : 0);
}
__host__ __device__ __forceinline__ long long hx_cta_begin(long long T, int n_cta, int c) {
  return c >= n_cta ? T : T * c / n_cta;
}
// the CTA whose range holds unit u: the largest c with cta_begin(c) <= u
__host__ __device__ __forceinline__ int hx_cta_of(long long T, int n_cta, long long u) {
  return (int)(((u + 1) * n_cta - 1) / T);
}

// Fixed-point strip sums: exact integer additions make the result independent of the order in
// which warps and CTAs contribute (deterministic), at 2^-32 resolution and +-2^22 range.
__device__ __forceinline__ unsigned long long hx_fix(float v) {
  if (!(fabsf(v) < LR_MAX)) {
    raise_flag(GSDLQ_FLAG_RANGE);
    v = (v != v) ? 0.f : copysignf(LR_MAX, v);
  }
  return (unsigned long long)__float2ll_rn(v * LR_FIX);
}
__device__ __forceinline__ float hx_unfix(unsigned long long a) {
  return (float)((double)(long long)a * (1.0 / 4294967296.0));
}

// Strips shared between CTAs.  Every CTA holding units of such a strip adds its fixed-point part
// plus HX_SH_ONE to the strip's global word of each row with one returning atomic per word.  A word
// thus carries the number of contributions in its top bits (at most 7, which the planner
// guarantees) and their sum below (|sum| < 2^59, far beyond the +-2^22 value range): the CTA whose
// addition completes word 0 finishes the strip, from the values its own atomics returned, without
// a separate counter or a second round trip.
constexpr unsigned long long HX_SH_ONE = 1ull << 60;
__device__ __forceinline__ unsigned hx_sh_count(unsigned long long w) { return (unsigned)((w + (HX_SH_ONE >> 1)) >> 60); }

inline size_t hexmv_ws_bytes_for(int n_strips, int nmat) {
  return ((sizeof(unsigned) * (CTL_WORDS + (size_t)n_strips) + 15) & ~size_t(15)) +
         sizeof(unsigned long long) * (size_t)n_strips * nmat * 16 + 256;
}

// ---- shared memory --------------------------------------------------------------------
// The decode table sits at the fixed shared-window address HX_TAB_ABS: one byte permute builds
// (code << 8 | lane << 2) from a code byte and the lane, and the lookup's load adds HX_TAB_ABS as
// its immediate offset.  Dynamic shared memory starts at a small offset B (the system-reserved
// bytes) below it:
//   [B, HX_TAB_ABS)                          reduction words (the last 256 bytes)
//   [HX_TAB_ABS, HX_TAB_ABS + 64 KB)         256 table rows of 256 bytes: 32 lanes x 4-byte
//                                            entries, then a free 128-byte half
//   [HX_TAB_ABS + 64 KB, ...)                activation-split overflow chunks
// The whole footprint stays small (68 KB for rows of up to 8192 columns) because shared memory
// taken from the unified L1 leaves less room for the code loads in flight.  The host sizes the
// allocation for B = 0; the kernel checks B and raises GSDLQ_FLAG_UNSUPPORTED if its reduction
// words would not fit below the table.
constexpr uint32_t HX_TAB_ABS = 0x1000u;
constexpr int HX_RED_BYTES = 2048;
constexpr int HX_LR_FLAG = 60;  // index (in the shared tmp_k area) of its ready flag

inline int hx_dyn_smem(int ovf_bytes) { return (int)HX_TAB_ABS + 0x10000 + ovf_bytes; }

// TMA ring (FULL streams with room for it): two slots per streaming warp right after the
// activation overflow; a slot holds one unit -- its four 64-byte code segments as 16 x 64-byte
// tiles (segment-major, so the 8 lanes of a quarter-warp read 128 contiguous bytes) and its 16
// rows of 8 fp16 scales.  The slots' mbarriers and (in the decode kernel) each warp's parity bits
// sit in the reduction words.
constexpr int HX_SLOT = 4 * 1024 + 256;
constexpr int HX_RING_BYTES = HX_STREAM * 2 * HX_SLOT;
constexpr int HX_MBAR_OFF = 1536;  // byte offset in the reduction words: 2 x 8 bytes per warp
constexpr int HX_PH_OFF = 1792;    // byte offset: one parity word per warp
inline int hx_dyn_smem_tma(int ovf_bytes) { return hx_dyn_smem(ovf_bytes) + HX_RING_BYTES; }
// the CTA's strip accumulator (placed at lacc_off, after the overflow chunks / the ring)
inline int hx_lacc_bytes(const HexmvParams& P) { return P.n_local * P.nmat * 16 * 8; }

// Activation splits.  For pair p (columns 2p, 2p+1) with a = x[2p], b = x[2p]/2 + sqrt3/2 x[2p+1],
// the hi word (bf16 a_hi | b_hi << 16) and the lo word live in 128-byte chunk
// ch = (p / 64) * 4 + (p % 16) / 4 at byte ((p % 64) / 16) * 32 + (p % 4) * 4 (+16 for lo).
// One chunk is exactly what the 32 lanes of a warp read with one 16-byte load per k-step
// pair, conflict-free.  The first 256 chunks fill the free halves of the table rows.
__device__ __forceinline__ uint32_t xs_chunk(int ch, uint32_t tab_off) {
  return ch < 256 ? tab_off + (uint32_t)ch * 256u + 128u : tab_off + 0x10000u + (uint32_t)(ch - 256) * 128u;
}

// ---- decode table ----------------------------------------------------------------------
// bf16 bits of a small integer (|v| <= 255: exact)
constexpr uint32_t bf16_of_int(int v) {
  if (v == 0) return 0u;
  const uint32_t sign = v < 0 ? 0x8000u : 0u;
  const int a = v < 0 ? -v : v;
  int e = 0;
  while ((a >> (e + 1)) != 0) ++e;  // floor(log2 a) <= 7
  return sign | ((uint32_t)(127 + e) << 7) | (((uint32_t)a << (7 - e)) & 0x7fu);
}
// The decode-table entries of both radii, made at compile time: entry c of radius R is the bf16x2
// (r0 low, r1 high) of the c-th point of the reference's enumeration (r0 outer, r1 inner,
// |r0 + r1| <= R; gsd_lq_cpu_runtime.py:111-118); codes past the last point decode to (0, 0).
struct LatticeEntries {
  uint32_t e[2][256];  // [0]: radius 6, [1]: radius 8
};
constexpr LatticeEntries make_lattice_entries() {
  LatticeEntries t{};
  for (int ri = 0; ri < 2; ++ri) {
    const int R = ri ? 8 : 6;
    int c = 0;
    for (int a = -R; a <= R; ++a)
      for (int b = -R; b <= R; ++b)
        if (a + b <= R && a + b >= -R) t.e[ri][c++] = bf16_of_int(a) | (bf16_of_int(b) << 16);
  }
  return t;
}
__device__ const LatticeEntries g_lattice_entries = make_lattice_entries();

// decode entry of code i from a caller's float xy table (the drop-in path); the table must be
// the A2 lattice, which is checked
__device__ __forceinline__ uint32_t entry_from_xy(const float* xy, int n_pts, int i) {
  if (i >= n_pts) return 0u;
  const float x = xy[2 * i], y = xy[2 * i + 1];
  const float rf1 = rintf(y * 1.1547005383792515f);
  const float rf0 = x - 0.5f * rf1;
  const float yy = (float)((double)rf1 * 0.8660254037844386);
  if (rf0 != rintf(rf0) || yy != y || fabsf(rf0) > 16.f || fabsf(rf1) > 16.f) {
    raise_flag(GSDLQ_FLAG_BAD_TABLE);
    return 0u;
  }
  return pack_bf16x2(rf0, rf1);
}

// Decode lookup: PRMT assembles code << 8 | lane << 2 (lane4x = lane*4 supplies byte 0 and the
// zero bytes 2, 3), and one 32-bit shared load at that address + HX_TAB_ABS reads the entry.
// The load is not volatile (the table is constant after the prologue barrier), so lookups can
// be scheduled around the MMAs; lane4x is derived from a shared-memory read made after that
// barrier, which keeps every lookup behind it.
__device__ __forceinline__ uint32_t tab_lookup(uint32_t word, uint32_t lane4x, uint32_t sel) {
  const uint32_t addr = __byte_perm(word, lane4x, sel);
  uint32_t r;
  asm("ld.shared.b32 %0, [%1+%2];" : "=r"(r) : "r"(addr), "n"(HX_TAB_ABS));
  return r;
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 r;
  asm("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}

// One 64-byte segment of a unit (16 rows x 64 code pairs = scale groups A and B): 8 MMAs in
// two independent accumulator chains.  ca / cb: this lane's 16 code bytes of rows g and g+8;
// baddr: this lane's 16-byte B slice in the segment's first chunk (chunks bstride apart).
// Only the 8 lanes whose B column has data on their own k rows load (bld); the B registers of
// the others were zeroed once and are never written, so the block-diagonal zeros cost nothing.
// Returns the dot products of this lane's group (q = 0: A, q = 1: B; 0 for q = 2, 3).
__device__ __forceinline__ void segment_mma(const uint4& ca, const uint4& cb, uint32_t baddr, uint32_t bstride,
                                            bool bld, uint4 (&bv)[2], uint32_t lane4x, float& r_g, float& r_h) {
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t wa[4] = {ca.x, ca.y, ca.z, ca.w};
  const uint32_t wb[4] = {cb.x, cb.y, cb.z, cb.w};
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    // k-steps 2m (code bytes 0, 1 of word m) and 2m+1 (bytes 2, 3)
    if (bld) bv[m & 1] = lds_u4(baddr + (uint32_t)m * bstride);
    uint32_t a0[4], a1[4];
    a0[0] = tab_lookup(wa[m], lane4x, 0x6504u);  // row g,   pair 2t
    a0[1] = tab_lookup(wb[m], lane4x, 0x6504u);  // row g+8, pair 2t
    a0[2] = tab_lookup(wa[m], lane4x, 0x6514u);  // row g,   pair 2t+1
    a0[3] = tab_lookup(wb[m], lane4x, 0x6514u);  // row g+8, pair 2t+1
    a1[0] = tab_lookup(wa[m], lane4x, 0x6524u);
    a1[1] = tab_lookup(wb[m], lane4x, 0x6524u);
    a1[2] = tab_lookup(wa[m], lane4x, 0x6534u);
    a1[3] = tab_lookup(wb[m], lane4x, 0x6534u);
    mma_bf16_16816(d0, a0, bv[m & 1].x, bv[m & 1].y, d0);
    mma_bf16_16816(d1, a1, bv[m & 1].z, bv[m & 1].w, d1);
  }
  r_g = (d0[0] + d0[1]) + (d1[0] + d1[1]);
  r_h = (d0[2] + d0[3]) + (d1[2] + d1[3]);
}

__device__ __forceinline__ unsigned long long ld_cg_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// bounded spin (1 s of %globaltimer) until a shared-memory flag set by another warp of the CTA is
// nonzero; on timeout the flag is raised and the caller continues
__device__ __forceinline__ void wait_shared_flag(const volatile float* flag, int lane) {
  if (*flag != 0.f) return;
  unsigned long long t0, t1;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (*flag == 0.f) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > 1000000000ull) {
      if (lane == 0) raise_flag(GSDLQ_FLAG_TIMEOUT);
      return;
    }
    __nanosleep(64);
  }
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

// Operands of a strip's epilogue that do not depend on its result, loaded before the CTA barrier
// so that their latency overlaps it.
struct EpiPre {
  float resid;  // RESID
  float2 cs;    // ROPE_KV: (cos, sin) of this row's pair at the current position
};

template <int EPI>
__device__ __forceinline__ EpiPre epilogue_pre(const HexmvParams& P, const StripInfo& si, int lane, int pos) {
  const gsdlq_linear_job_t& J = P.job;
  EpiPre e{0.f, make_float2(1.f, 0.f)};
  const int row = si.rbase + (lane & 15);
  const bool ok = lane < 16 && row < J.mat[si.m0].rows;
  if constexpr (EPI == GSDLQ_EPI_RESID) {
    if (ok) e.resid = __ldcg(J.resid + row);
  } else if constexpr (EPI == GSDLQ_EPI_ROPE_KV) {
    if (ok && si.m0 != 2 && pos >= 0 && pos < J.max_seq) {
      const int hd = J.head_dim;
      e.cs = __ldg(reinterpret_cast<const float2*>(J.rope_cs) + (size_t)pos * (hd / 2) + ((row % hd) >> 1));
    }
  }
  return e;
}

// Epilogue of a completed strip.  Lane j holds the finished value of row (j & 15) of
// matrix m0 + (j >> 4) (lanes >= 16 only carry data in pair mode).  Returns, in lanes 0-15, the
// value written for the row (the next linear's input; 0 for ROPE_KV and rows past the end).
template <int EPI>
__device__ float strip_epilogue(const HexmvParams& P, const StripInfo& si, float v, int lane, const EpiPre& pre,
                                int pos, int layer) {
  const gsdlq_linear_job_t& J = P.job;
  const int r = lane & 15;
  const gsdlq_hexmat_t& M = J.mat[si.m0];
  const int row = si.rbase + r;
  const bool ok = row < M.rows;
  float out = 0.f;
  if constexpr (EPI == GSDLQ_EPI_STORE) {
    unsigned long long key = 0ull;
    if (lane < 16 && ok) {
      J.y[si.m0][row] = v;
      out = v;
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
    if (lane < 16 && ok) {
      out = pre.resid + v;
      J.y[0][row] = out;
    }
  } else if constexpr (EPI == GSDLQ_EPI_SWIGLU) {
    const float u = __shfl_down_sync(0xffffffffu, v, 16);
    if (lane < 16 && ok) {
      out = (v / (1.0f + expf(-v))) * u;
      J.y[0][row] = out;
    }
  } else if constexpr (EPI == GSDLQ_EPI_ROPE_KV) {
    // rows (2i, 2i+1) of a head form one interleaved RoPE pair
    const float other = __shfl_xor_sync(0xffffffffu, v, 1);
    if (lane < 16 && ok) {
      const bool even = (r & 1) == 0;
      const float v0 = even ? v : other, v1 = even ? other : v;
      const bool pos_ok = pos >= 0 && pos < J.max_seq;
      if (!pos_ok && lane == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
      if (si.m0 == 2) {  // V: stored unrotated
        if (J.y[2]) J.y[2][row] = v;
        if (pos_ok) J.v_cache[((size_t)layer * J.max_seq + pos) * M.rows + row] = f2h(v);
      } else {
        const float2 cs = pre.cs;
        const float o = even ? __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y))
                             : __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
        if (si.m0 == 0) {
          J.y[0][row] = o;
        } else {
          if (J.y[1]) J.y[1][row] = o;
          if (pos_ok) J.k_cache[((size_t)layer * J.max_seq + pos) * M.rows + row] = f2h(o);
        }
      }
    }
  }
  return out;
}

// Low-rank forwarding (job.fwd_acc): this strip's 16 output rows r contribute
// sum_r Vt_next[j][rbase + r] * w[rbase + r] * out_r to the next linear's accumulator j.  Lane l
// handles accumulators l and l + 32; their Vt slices (16 fp16 each) are loaded before the strip's
// CTA barrier so that the loads overlap it.
struct FwdSlice {
  uint4 a[2], b[2];
  float w;  // lanes 0-15: the next linear's norm weight of row rbase + lane (1 without one)
};
__device__ __forceinline__ int fwd_total(const gsdlq_linear_job_t& J) { return J.fwd_k[0] + J.fwd_k[1] + J.fwd_k[2]; }
__device__ __forceinline__ const uint16_t* fwd_row(const gsdlq_linear_job_t& J, int jl, int n_out) {
  int m = 0, j = jl;
  while (m < 2 && j >= J.fwd_k[m]) j -= J.fwd_k[m], ++m;
  return J.fwd_vt[m] + (size_t)j * n_out;
}
__device__ __forceinline__ FwdSlice fwd_load(const gsdlq_linear_job_t& J, int rbase, int n_out, int lane) {
  FwdSlice f;
  const int nk = fwd_total(J);
  const int row = rbase + (lane & 15);
  f.w = (J.fwd_norm_w != nullptr && lane < 16 && row < n_out) ? __ldg(J.fwd_norm_w + row) : 1.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int jl = lane + 32 * h;
    const bool whole = rbase + 16 <= n_out;  // (n_out is a multiple of 64: strips never straddle it)
    if (jl < nk && whole) {
      const uint4* v = reinterpret_cast<const uint4*>(fwd_row(J, jl, n_out) + rbase);
      f.a[h] = __ldg(v);
      f.b[h] = __ldg(v + 1);
    } else {
      f.a[h] = make_uint4(0u, 0u, 0u, 0u);
      f.b[h] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  return f;
}
__device__ __forceinline__ float fwd_dot16(const uint4& a, const uint4& b, float o, int lane) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float acc = 0.f;
#pragma unroll
  for (int r = 0; r < 16; ++r) acc = fmaf(h2f((uint16_t)(w[r >> 1] >> (16 * (r & 1)))), __shfl_sync(0xffffffffu, o, r), acc);
  (void)lane;
  return acc;
}
__device__ __forceinline__ void fwd_apply(const gsdlq_linear_job_t& J, const FwdSlice& f, int rbase, int n_out, float out,
                                          int lane) {
  const int row = rbase + (lane & 15);
  const float o = (lane < 16 && row < n_out) ? out * f.w : 0.f;
  const int nk = fwd_total(J);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (32 * h >= nk) break;  // uniform
    float acc = fwd_dot16(f.a[h], f.b[h], o, lane);
    const int jl = lane + 32 * h;
    if (jl < nk) {
      if (!(fabsf(acc) < LR_MAX)) {
        raise_flag(GSDLQ_FLAG_RANGE);
        acc = (acc != acc) ? 0.f : copysignf(LR_MAX, acc);
      }
      atomicAdd(J.fwd_acc + jl, (unsigned long long)__float2ll_rn(acc * LR_FIX));
    }
  }
}

// Epilogue of a completed strip whose final sum v lane j holds (row j & 15 of matrix
// m0 + (j >> 4)), with low-rank forwarding (one warp).
// The operands of a strip's epilogue that do not depend on its sum (loaded ahead of it).
struct StripPre {
  EpiPre e;
  FwdSlice f;
};
template <int EPI>
__device__ __forceinline__ StripPre strip_pre(const HexmvParams& P, const StripInfo& si, int lane, int pos) {
  StripPre sp;
  sp.e = epilogue_pre<EPI>(P, si, lane, pos);
  if (P.job.fwd_acc != nullptr) sp.f = fwd_load(P.job, si.rbase, P.job.mat[si.m0].rows, lane);
  return sp;
}
template <int EPI, int NMAT, class PTR>
__device__ __forceinline__ void finish_value(const HexmvParams& P, const PTR& mp, const StripInfo& si, float v, int lane,
                                             int pos, const StripPre& sp) {
  const int n_out = P.job.mat[si.m0].rows;
  const float out = strip_epilogue<EPI>(P, si, v, lane, sp.e, pos, mp.layer());
  if (P.job.fwd_acc != nullptr) fwd_apply(P.job, sp.f, si.rbase, n_out, out, lane);
}

// After a CTA's last helper warp has read the low-rank accumulators: count it; the last CTA of
// the launch leaves every control word at zero for the workspace's next user (its acquire
// orders the zeroing after every CTA's reads, which precede their releases of the count).
__device__ __forceinline__ void ctl_release_last(unsigned* ctl, int lane) {
  unsigned last = 0u;
  if (lane == 0) last = atom_add_acq_rel(&ctl[CTL_DONE], 1u) == gridDim.x - 1 ? 1u : 0u;
  if (__shfl_sync(0xffffffffu, last, 0)) {
    for (int i = lane; i < CTL_WORDS; i += 32) ctl[i] = 0u;
  }
}

// The whole fused linear for one CTA.  MEGA = false: a stand-alone launch (programmatic dependent
// launch, the decode table built here, the control words reset by the last CTA).  MEGA = true: one
// phase of the persistent decode kernel, which built the table once (s_radius in the reduction
// words holds its radius) and orders the phases through the accessor's dep / done counters.
template <int EPI, bool FULL, bool MEGA, bool TMA, class PTR, bool UK = true>
__device__ __forceinline__ void hexmv_body(const HexmvParams& P, const PTR& mp, uint8_t* smem) {
  static_assert(!TMA || FULL, "the TMA ring streams whole units only");
  // per-unit kink lists are applied by the streaming warps of the per-lane-load paths only; the host
  // never picks the TMA ring for a launch that has them
  // UK = false compiles the per-unit kink path out (it costs the streaming loop registers and code)
  const bool ukink = UK && !TMA && P.ukink;
  constexpr int NMAT = (EPI == GSDLQ_EPI_SWIGLU) ? 2 : 1;
  constexpr int width = NMAT * 16;
  const gsdlq_linear_job_t& J = P.job;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gl = lane >> 2, q = lane & 3;
  const int C = P.cols, G = P.G, NP = P.NP;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  if (sbase + HX_RED_BYTES > HX_TAB_ABS || (sbase & 15u)) {  // the layout's assumption on the reserved bytes
    if (tid == 0) {
      raise_flag(GSDLQ_FLAG_UNSUPPORTED);
      if (mp.abort()) atomicExch(mp.abort(), 1u);
    }
    return;
  }
  // the next launch may be scheduled at once: its CTAs take an SM as soon as one of ours leaves it,
  // and its griddepcontrol.wait still waits for this whole grid
  if (!MEGA) pdl_launch_dependents();
#ifdef GSDLQ_TRACE
  if (tid == 0) {
    unsigned slot;
    if constexpr (MEGA) slot = mp.trace_slot();  // the phase index inside the persistent step
    else slot = atomicAdd(&g_trace_cnt[blockIdx.x], 1u);
    reinterpret_cast<uint32_t*>(smem + (HX_TAB_ABS - sbase) - HX_RED_BYTES)[40] = slot;
    GSDLQ_TR_SET(slot, 0, tr_now());
    GSDLQ_TR_SET(slot, 9, ((unsigned long long)P.job.layer << 8) | (unsigned)P.job.epilogue);
  }
#define HX_SLOT_NOW (reinterpret_cast<const volatile uint32_t*>(smem + (HX_TAB_ABS - sbase) - HX_RED_BYTES)[40])
#else
#define HX_SLOT_NOW 0u
#endif
  const uint32_t tab_off = HX_TAB_ABS - sbase;
  uint8_t* tab = smem + tab_off;
  float* red = reinterpret_cast<float*>(smem + tab_off - HX_RED_BYTES);
  // [1..16] warp sums, [32] [33] zero words, [34] position, [35] radius (decode kernel), [37] 1/rms,
  // [38] finished strips; s_lr: [0..48) tmp_k, [HX_LR_FLAG] ready; then 16 kink row sums per
  // streaming warp
  volatile float* s_lr = red + 64;
  float* s_ks = red + 128 + 16 * warp;
  // (x[2p], x[2p+1]) recovered from the staged splits (hi + lo: about 16 significant bits)
  auto xs_pair = [&](int p) -> float2 {
    const int j = p & 63, r = j & 15;
    const uint32_t off = xs_chunk((p >> 6) * 4 + (r >> 2), tab_off) + (uint32_t)((j >> 4) * 32 + (r & 3) * 4);
    const uint32_t h = *reinterpret_cast<const uint32_t*>(smem + off);
    const uint32_t l = *reinterpret_cast<const uint32_t*>(smem + off + 16);
    const float x0 = bf16lo_to_f(h) + bf16lo_to_f(l);
    const float b = bf16hi_to_f(h) + bf16hi_to_f(l);
    return make_float2(x0, (b - 0.5f * x0) * 1.1547005383792515f);
  };
  uint32_t* redu = reinterpret_cast<uint32_t*>(red);
  // this CTA's unit range, the strips it touches [s_lo, s_hi] and their fixed-point sums
  const long long cb0 = hx_cta_begin(P.T, P.n_cta, blockIdx.x), cb1 = hx_cta_begin(P.T, P.n_cta, blockIdx.x + 1);
  const int s_lo = (int)(cb0 / P.UPS), s_hi = cb1 > cb0 ? (int)((cb1 - 1) / P.UPS) : s_lo - 1;
  unsigned long long* lacc = reinterpret_cast<unsigned long long*>(smem + tab_off + P.lacc_off);

  // Barriers: 0 = the whole CTA (end only); 1 = the 14 streaming warps; 2 = streaming warps
  // arrive once the input is staged, helper warps wait on it only when they need the input.
  const bool helper = warp >= HX_STREAM;
  constexpr int NST = HX_STREAM * kWarp;  // streaming (and staging) threads

  if (helper) {
    // ==== helper warps: low-rank slice partials and the kink sums of the strips this CTA owns ===
    // the later launches' weights go into L2 first, while this launch waits for its input
    if (!MEGA && warp == HX_STREAM) issue_prefetch(J.prefetch, blockIdx.x, gridDim.x, lane);
    const int hw = blockIdx.x * HX_HELP + (warp - HX_STREAM);
    const int H = gridDim.x * HX_HELP;
    const int c8_0 = hw * P.lr_chunks;
    const int c8_1 = min(c8_0 + P.lr_chunks, C / 8);
    constexpr int SPP = (NMAT == 2) ? 1 : 2;  // strips per kink pass
    // The kink and low-rank terms of the strips this CTA owns (those whose first unit is in its
    // range) go into its accumulator; pass p of helper warp hl covers strip
    // o_lo + (p * HX_HELP + hl) * SPP (+ 1 for lanes 16-31 when SPP == 2); lane = row.
    const int hl = warp - HX_STREAM;
    const int o_lo = cb1 > cb0 ? (int)((cb0 + P.UPS - 1) / P.UPS) : 0;
    const int o_hi = cb1 > cb0 ? (int)((cb1 + P.UPS - 1) / P.UPS) : 0;
    auto pass_strip = [&](int p) { return o_lo + (p * HX_HELP + hl) * SPP + ((NMAT == 2) ? 0 : (lane >> 4)); };
    const int npass = o_hi > o_lo + hl * SPP ? (o_hi - o_lo - hl * SPP + HX_HELP * SPP - 1) / (HX_HELP * SPP) : 0;
    (void)H;
    struct KRow {
      const uint16_t* cols;
      const float* del;
      uint32_t e0, e1;
      int km, row;  // matrix and row of this lane (row -1: none)
    };
    // row offsets and kink arrays of this lane's row in pass p (copied out of the parameters)
    auto krow = [&](int p) -> KRow {
      KRow k{nullptr, nullptr, 0u, 0u, 0, -1};
      const int s = pass_strip(p);
      if (p < npass && s < o_hi) {
        const StripInfo si = strip_info<NMAT>(P, s);
        const int km = si.m0 + ((NMAT == 2) ? (lane >> 4) : 0);
        k.km = km;
        k.cols = mp.mat(km).kink_cols;
        k.del = mp.mat(km).kink_deltas;
        const int row = si.rbase + (lane & 15);
        if (row < J.mat[km].rows) {
          k.row = row;
          if (!ukink) {  // otherwise the streaming warps apply the kinks
            const uint32_t* rp = mp.mat(km).row_ptr;
            k.e0 = __ldg(rp + row);
            k.e1 = __ldg(rp + row + 1);
          }
        }
      }
      return k;
    };
    // L2 prefetch of the kink columns and deltas of a pass's rows, so that the pass's batches hit L2
    // instead of queueing behind the streaming warps' HBM loads
    auto pf_kinks = [&](const KRow& k) {
      if (k.row >= 0 && k.e1 > k.e0) {
        const uint8_t* c = reinterpret_cast<const uint8_t*>(k.cols + k.e0);
        const uint8_t* d = reinterpret_cast<const uint8_t*>(k.del + k.e0);
        for (uint32_t b = 0; b < (k.e1 - k.e0) * 2u + 127u; b += 128u) asm volatile("prefetch.global.L2 [%0];" ::"l"(c + b));
        for (uint32_t b = 0; b < (k.e1 - k.e0) * 4u + 127u; b += 128u) asm volatile("prefetch.global.L2 [%0];" ::"l"(d + b));
      }
    };
    constexpr int KB = 8;  // kinks per lane per batch
    int col[KB];
    float dl[KB];
    auto load_batch = [&](const KRow& k, uint32_t e) {
#pragma unroll
      for (int u = 0; u < KB; ++u) {
        const uint32_t eu = e + u;
        col[u] = eu < k.e1 ? (int)__ldg(k.cols + eu) : 0;
        dl[u] = eu < k.e1 ? __ldg(k.del + eu) : 0.f;
      }
    };
    // the U row of this lane's row in the pass (raw fp16 bits), loaded with the pass's first batch
    uint16_t ur[16];
    auto load_u = [&](const KRow& k) {
      const int kd = k.row >= 0 ? J.mat[k.km].k_dim : 0;
      const uint16_t* up = mp.mat(k.km).U + (size_t)(k.row < 0 ? 0 : k.row) * kd;
#pragma unroll
      for (int j = 0; j < 16; ++j) ur[j] = j < kd ? __ldg(up + j) : (uint16_t)0;
    };
    // ---- before the wait: everything that does not depend on x -----------------------------
    KRow kcur = krow(0), knext = krow(1);
    load_batch(kcur, kcur.e0);
    load_u(kcur);
    pf_kinks(kcur);
    pf_kinks(knext);
    constexpr int LRC = 4;  // Vt chunks of this lane's first row held in registers; the rest via L2
    uint4 vr[LRC];
    auto vt_row = [&](int jl) {  // Vt row jl of the launch's concatenated low-rank rows
      int m = 0, j = jl;
      while (m < J.n_mat - 1 && j >= J.mat[m].k_dim) j -= J.mat[m].k_dim, ++m;
      return reinterpret_cast<const uint4*>(mp.mat(m).Vt + (size_t)j * C);
    };
    const bool lr_here = P.n_lr > 0 && !J.lr_forwarded;  // else the previous launch forwarded it
#pragma unroll 1
    for (int jl = lane; lr_here && jl < P.n_lr; jl += 32) {
      const uint4* vt = vt_row(jl);
      if (jl == lane) {
#pragma unroll
        for (int k = 0; k < LRC; ++k) vr[k] = (c8_0 + k < c8_1) ? __ldg(vt + c8_0 + k) : make_uint4(0u, 0u, 0u, 0u);
      }
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(vt);
      for (int b = ((c8_0 + (jl == lane ? LRC : 0)) * 16) & ~127; b < c8_1 * 16; b += 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + b));
    }
    // ---- the staged input, and the previous kernel's outputs, are ready after these ------------
    named_bar_sync(2, HX_THREADS);
    if (!MEGA) pdl_wait();  // (in the decode kernel the staging threads' acquire precedes barrier 2)
    const int pos = reinterpret_cast<const int*>(redu)[34];
    // the input values come back from the staged splits (xs_pair), so no fp32 copy of x occupies
    // shared memory and no gather waits on L2
    auto dot8 = [&](const uint4& raw, int c8) {  // 8 columns of one Vt row against x
      const float2 a0 = xs_pair(4 * c8), a1 = xs_pair(4 * c8 + 1), a2 = xs_pair(4 * c8 + 2), a3 = xs_pair(4 * c8 + 3);
      return a0.x * h2f(raw.x & 0xffffu) + a0.y * h2f(raw.x >> 16) + a1.x * h2f(raw.y & 0xffffu) +
             a1.y * h2f(raw.y >> 16) + a2.x * h2f(raw.z & 0xffffu) + a2.y * h2f(raw.z >> 16) +
             a3.x * h2f(raw.w & 0xffffu) + a3.y * h2f(raw.w >> 16);
    };
    if (P.n_lr > 0 && J.lr_forwarded) {
      // the previous launch added every row's term: scale by S (the 1/rms of a normed input is applied
      // to the finished strip values)
      if (warp == HX_WARPS - 1) {
        const unsigned long long* acc = reinterpret_cast<const unsigned long long*>(mp.ctl() + CTL_TMPK);
        for (int jl = lane; jl < P.n_lr; jl += 32) {
          int m = 0, j = jl;
          while (m < J.n_mat - 1 && j >= J.mat[m].k_dim) j -= J.mat[m].k_dim, ++m;
          const double d = (double)(long long)__ldcg(acc + jl) * (1.0 / 4294967296.0);
          s_lr[jl] = (float)d * __ldg(mp.mat(m).S + j);
        }
        __threadfence_block();
        __syncwarp();
        if (lane == 0) s_lr[HX_LR_FLAG] = 1.f;
        ctl_release_last(mp.ctl(), lane);
      }
    } else if (P.n_lr > 0) {
#pragma unroll 1
      for (int jl = lane; jl - lane < P.n_lr; jl += 32) {  // uniform trip count: all lanes reach the fence
        if (jl < P.n_lr) {
          const uint4* vt = vt_row(jl);
          const bool first = jl == lane;
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < LRC; ++k)
            if (c8_0 + k < c8_1) acc += dot8(first ? vr[k] : __ldg(vt + c8_0 + k), c8_0 + k);
          for (int cb = c8_0 + LRC; cb < c8_1; cb += 4) {
            uint4 raw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) raw[k] = (cb + k < c8_1) ? __ldg(vt + cb + k) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (cb + k < c8_1) acc += dot8(raw[k], cb + k);
          }
          if (!(fabsf(acc) < LR_MAX)) {
            raise_flag(GSDLQ_FLAG_RANGE);
            acc = (acc != acc) ? 0.f : copysignf(LR_MAX, acc);
          }
          const long long fx = __float2ll_rn(acc * LR_FIX);
          atomicAdd(reinterpret_cast<unsigned long long*>(mp.ctl() + CTL_TMPK) + jl, (unsigned long long)fx);
        }
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(&mp.ctl()[CTL_LR_DONE], 1u);
      if (warp == HX_WARPS - 1) {
        // once every slice is in, publish S * projection to this CTA's finishing warps
        if (lane == 0) wait_eq_abort(&mp.ctl()[CTL_LR_DONE], gridDim.x * HX_HELP, mp.abort());  // 1 s bound
        __syncwarp();  // lane 0's acquire load orders the accumulator reads of the warp
        const unsigned long long* acc = reinterpret_cast<const unsigned long long*>(mp.ctl() + CTL_TMPK);
        for (int jl = lane; jl < P.n_lr; jl += 32) {
          int m = 0, j = jl;
          while (m < J.n_mat - 1 && j >= J.mat[m].k_dim) j -= J.mat[m].k_dim, ++m;
          const double d = (double)(long long)__ldcg(acc + jl) * (1.0 / 4294967296.0);
          s_lr[jl] = (float)d * __ldg(mp.mat(m).S + j);
        }
        __threadfence_block();
        __syncwarp();
        if (lane == 0) s_lr[HX_LR_FLAG] = 1.f;
        ctl_release_last(mp.ctl(), lane);
        if (lane == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 14, tr_now());
      }
    }
    // ---- kink passes: one slot per strip; the counts are made together at the end -------------
    bool bad = false;
    for (int p = 0; p < npass; ++p) {
      if (p > 0) {
        kcur = knext;
        knext = krow(p + 1);  // in flight during this pass
        load_batch(kcur, kcur.e0);
        load_u(kcur);
        pf_kinks(knext);  // waits for its row offsets, which overlaps this pass's first batch
      }
      float v = 0.f;
      for (uint32_t e = kcur.e0;;) {
#pragma unroll
        for (int u = 0; u < KB; ++u) {
          const bool in = e + u < kcur.e1;
          const bool ok = col[u] < C;
          if (in && ok) {
            const float2 xp = xs_pair(col[u] >> 1);
            v += dl[u] * ((col[u] & 1) ? xp.y : xp.x);
          }
          bad |= in && !ok;
        }
        e += KB;
        if (!__any_sync(0xffffffffu, e < kcur.e1)) break;
        load_batch(kcur, e);
      }
      // the low-rank term: U row . tmp_k, tmp_k from this CTA's shared copy (or the caller's)
      const int kd = kcur.row >= 0 ? J.mat[kcur.km].k_dim : 0;
      if (__any_sync(0xffffffffu, kd > 0)) {
        float lr = 0.f;
        if (P.tmp_k_ext != nullptr) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < kd) lr += h2f(ur[j]) * __ldg(P.tmp_k_ext + j);
        } else {
          wait_shared_flag(s_lr + HX_LR_FLAG, lane);
          const volatile float* tk = s_lr + P.lr_off[kcur.km];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < kd) lr += h2f(ur[j]) * tk[j];
        }
        v += lr;
      }
      const int s = pass_strip(p);
      if (s < o_hi) atomicAdd(lacc + (size_t)(s - s_lo) * width + (lane & (width - 1)), hx_fix(v));
    }
    if (bad) raise_flag(GSDLQ_FLAG_BAD_KINK);
    if (lane == 0) GSDLQ_TR_MAX(HX_SLOT_NOW, 8);
  } else {
    // ==== streaming warps ===================================================================
    if (lane < 16) s_ks[lane] = 0.f;
    const bool streamer = cb1 > cb0;
    const long long n_c = cb1 - cb0;
    // (unit indices and a CTA's range fit 32 bits: the planner keeps T below 2^31)
    const int u0 = (int)cb0 + (int)n_c * hx_lp(warp) / hx_lp(HX_STREAM);
    const int u1 = (int)cb0 + (int)n_c * hx_lp(warp + 1) / hx_lp(HX_STREAM);
    // cursor (strip, matrix in strip, unit column) of the next unit to load, and its pointers
    int ns = u0 / P.UPS;
    int nm = (u0 - ns * P.UPS) / P.GU;
    int nc = u0 - ns * P.UPS - nm * P.GU;
    const uint8_t* pa = nullptr;
    const uint8_t* pb = nullptr;
    const uint16_t* qa = nullptr;
    const uint16_t* qb = nullptr;
    auto seek = [&]() {
      const StripInfo si = strip_info<NMAT>(P, ns);
      const gsdlq_hexmat_t& M = mp.mat(si.m0 + nm);
      const int ra = min(si.rbase + gl, M.rows - 1), rb = min(si.rbase + gl + 8, M.rows - 1);
      pa = M.codes + (size_t)ra * NP + nc * HX_UB + q * 16;
      pb = M.codes + (size_t)rb * NP + nc * HX_UB + q * 16;
      qa = M.scales + (size_t)ra * G + nc * 8;
      qb = M.scales + (size_t)rb * G + nc * 8;
    };
    auto step_next = [&]() {  // the next unit: along the row, or the start of the next row block
      if (++nc == P.GU) {
        nc = 0;
        if (++nm == NMAT) {
          nm = 0;
          ++ns;
        }
        if (!TMA) seek();
      } else if (!TMA) {
        pa += HX_UB;
        pb += HX_UB;
        qa += 8;
        qb += 8;
      }
    };
    // the FULL path shifts the lane's fp16 scale out of a word holding two groups
    const int sh = FULL ? 16 * (q & 1) : 0;
    uint4 cw[4][2];         // code bytes of the unit being consumed / refilled: [segment][row g, g+8]
    uint32_t sa[4], sb[4];  // the next unit's scale words: [segment]
    uint32_t nko0 = 0u, nko1 = 0u;  // the next unit's kink range
    auto load_codes = [&](int s) {
      if (FULL || nc * HX_UB + 64 * s + 16 * q < NP) {
        cw[s][0] = ldg_stream_u4(pa + 64 * s);
        cw[s][1] = ldg_stream_u4(pb + 64 * s);
      } else {
        cw[s][0] = make_uint4(0u, 0u, 0u, 0u);  // past the row: its activations are staged as zero
        cw[s][1] = make_uint4(0u, 0u, 0u, 0u);
      }
    };
    auto load_scales = [&]() {
      if (ukink) {
        const StripInfo si = strip_info<NMAT>(P, ns);
        const uint32_t* kof = mp.mat(si.m0 + nm).unit_kink_off + (size_t)(si.rbase / 16) * P.GU + nc;
        nko0 = __ldg(kof);
        nko1 = __ldg(kof + 1);
      }
      if (TMA) {
        // the ring holds the scales
      } else if (FULL) {
        const uint4 x = ldg_stream_u4(qa), y = ldg_stream_u4(qb);
        sa[0] = x.x, sa[1] = x.y, sa[2] = x.z, sa[3] = x.w;
        sb[0] = y.x, sb[1] = y.y, sb[2] = y.z, sb[3] = y.w;
      } else {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const int gi = 2 * s + (q & 1);
          const bool ok = nc * 8 + gi < G;
          sa[s] = ok ? (uint32_t)__ldg(qa + gi) : 0u;
          sb[s] = ok ? (uint32_t)__ldg(qb + gi) : 0u;
        }
      }
    };
    // TMA ring: slot j of this warp holds unit u0 + i for i = j (mod 2); lane 0 issues the copies
    const uint32_t slot0 = sbase + tab_off + 0x10000u + (uint32_t)P.ovf_bytes + (uint32_t)(warp * 2 * HX_SLOT);
    const uint32_t bar0 = sbase + (tab_off - HX_RED_BYTES) + (uint32_t)(HX_MBAR_OFF + warp * 16);
    uint32_t* ph_word = reinterpret_cast<uint32_t*>(smem + (tab_off - HX_RED_BYTES) + HX_PH_OFF) + warp;
    uint32_t ph = 0u;  // parity of each slot's next phase (bit j: slot j)
    int is_ = ns, im_ = nm, ic_ = nc;  // issue cursor
    auto issue = [&](int slot) {  // lane 0: the unit at the issue cursor into `slot`
      const StripInfo si = strip_info<NMAT>(P, is_);
      const int mi = si.m0 + im_;
      const void* tc = mp.tmap_codes(mi);
      const void* ts = mp.tmap_scales(mi);
      const uint32_t dst = slot0 + (uint32_t)(slot * HX_SLOT), bar = bar0 + (uint32_t)(slot * 8);
      mbar_arrive_expect_tx(bar, (uint32_t)HX_SLOT);
#pragma unroll
      for (int k = 0; k < 4; ++k) tma_load_2d(dst + (uint32_t)(k * 1024), tc, ic_ * HX_UB + 64 * k, si.rbase, bar);
      tma_load_2d(dst + 4096u, ts, ic_ * 8, si.rbase, bar);
    };
    auto issue_next = [&]() {
      if (++ic_ == P.GU) {
        ic_ = 0;
        if (++im_ == NMAT) {
          im_ = 0;
          ++is_;
        }
      }
    };
    if (TMA && streamer) {
      if (!MEGA && lane == 0) {
        mbar_init(bar0, 1u);
        mbar_init(bar0 + 8u, 1u);
        mbar_fence_init();
      }
      if (MEGA) ph = *ph_word;
      __syncwarp();
    }
    // this thread's decode-table entry is loaded before the weight loads, so it does not queue behind them
    const bool build_table = !MEGA || reinterpret_cast<const volatile int*>(redu)[35] != J.mat[0].radius;
    const uint32_t tab_e = (build_table && tid < 256 && P.xy_table == nullptr)
                               ? __ldg(&g_lattice_entries.e[J.mat[0].radius == 8 ? 1 : 0][tid]) : 0u;
    if (streamer && u1 > u0) {
      if (TMA) {
        if (lane == 0) {
          issue(0);
          issue_next();
          if (u1 > u0 + 1) {
            issue(1);
            issue_next();
          }
        }
        if (ukink) load_scales();
      } else {
        seek();
        load_scales();
#pragma unroll
        for (int s = 0; s < 4; ++s) load_codes(s);
      }
    }

    // decode table (after the first unit's loads are in flight: it does not depend on them).  The
    // decode kernel keeps the table of the previous phase when the lattice radius is the same.
    if (build_table && P.xy_table != nullptr) {
      // the drop-in path: entries derived from the caller's float table (checked to be the lattice)
      for (int rb = warp * 16; rb < 256; rb += HX_STREAM * 16) {
        const uint32_t e = entry_from_xy(P.xy_table, P.n_pts, rb + (lane & 15));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t ek = __shfl_sync(0xffffffffu, e, 4 * k + (lane >> 3));
          const int row = rb + 4 * k + (lane >> 3);
          *reinterpret_cast<uint4*>(tab + row * 256 + (lane & 7) * 16) = make_uint4(ek, ek, ek, ek);
        }
      }
    } else if (build_table && tid < 256) {
      // thread t fills row t (the 32 per-lane copies of entry t) from the compile-time entries; its
      // 16-byte stores rotate through the row so that a warp's stores spread over all banks
      const uint4 v = make_uint4(tab_e, tab_e, tab_e, tab_e);
#pragma unroll
      for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(tab + tid * 256 + ((j + tid) & 7) * 16) = v;
    }
    if (tid == 0) {
      redu[32] = 0u;  // zero bits for the lookup addresses, read after a barrier
      redu[33] = 0u;
      s_lr[HX_LR_FLAG] = 0.f;
    }
    if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 10, tr_now());
    // the norm weights of this thread's first staging pairs do not depend on the producer: load them now
    constexpr int XR = 8;
    const bool normed = mp.input_mode() != GSDLQ_IN_PLAIN;
    float2 wpre[XR];
#pragma unroll
    for (int k = 0; k < XR; ++k) {
      const int p = tid + k * NST;
      wpre[k] = (normed && p < NP) ? __ldg(reinterpret_cast<const float2*>(mp.norm_w()) + p) : make_float2(1.f, 1.f);
    }
    // ---- wait for the producer of x, then stage the input ---------------------------------
    if (MEGA) {
      if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 1, tr_now());
      if (tid == 0 && mp.dep() != nullptr) wait_geq_abort(mp.dep(), mp.dep_target(), mp.abort());
      if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 2, tr_now());
      named_bar_sync(1, NST);
    } else {
      if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 1, tr_now());
      pdl_wait();
      if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 2, tr_now());
    }
    if (tid == 0) {
      int pv = -1;
      if (EPI == GSDLQ_EPI_ROPE_KV) pv = *J.pos;
      reinterpret_cast<int*>(redu)[34] = pv;
      // the call number of this launch's exchange (read by every CTA before the last one advances it)
      if (EPI == GSDLQ_EPI_RESID && !MEGA && P.ex_on) redu[41] = *reinterpret_cast<volatile unsigned*>(ex_words(P.ex)) + 1u;
    }
    int tok = 0;
    if (mp.input_mode() == GSDLQ_IN_EMBED) {
      tok = *J.token;
      if (tok < 0 || tok >= J.vocab) {
        if (tid == 0) raise_flag(GSDLQ_FLAG_BAD_TOKEN);
        tok = 0;
      }
    }
    auto load_x = [&](int p) -> float2 {
      if (mp.input_mode() == GSDLQ_IN_EMBED) {
        const uint32_t raw = __ldg(reinterpret_cast<const unsigned int*>(J.embed + (size_t)tok * C) + p);
        return make_float2(h2f(raw & 0xffffu), h2f(raw >> 16));
      }
      // .cg, not the non-coherent path: in the decode kernel x was written earlier in the same launch
      return __ldcg(reinterpret_cast<const float2*>(J.x) + p);
    };
    auto load_w = [&](int p) -> float2 {
      return normed ? __ldg(reinterpret_cast<const float2*>(mp.norm_w()) + p) : make_float2(1.f, 1.f);
    };
    auto stage = [&](int p, float x0, float x1, float2 wv, float inv) {
      if (mp.input_mode() == GSDLQ_IN_EMBED && blockIdx.x == 0 && J.x_out)
        reinterpret_cast<float2*>(J.x_out)[p] = make_float2(x0, x1);
      if (normed) {
        x0 = __fmul_rn(__fmul_rn(x0, inv), wv.x);
        x1 = __fmul_rn(__fmul_rn(x1, inv), wv.y);
      }
      const float b = fmaf(0.8660254037844386f, x1, 0.5f * x0);
      uint32_t h, l;
      split_bf16x2(x0, b, h, l);
      const int j = p & 63, r = j & 15;
      const uint32_t off = xs_chunk((p >> 6) * 4 + (r >> 2), tab_off) + (uint32_t)((j >> 4) * 32 + (r & 3) * 4);
      *reinterpret_cast<uint32_t*>(smem + off) = h;
      *reinterpret_cast<uint32_t*>(smem + off + 16) = l;
    };
    if (!normed) {
      // a plain input: batches of 2 XR pairs, so the 14336-wide down-projection input is staged
      // with one round of loads
      for (int p0 = tid; p0 < NP; p0 += 2 * XR * NST) {
        float2 t[2 * XR];
#pragma unroll
        for (int k = 0; k < 2 * XR; ++k) t[k] = (p0 + k * NST < NP) ? load_x(p0 + k * NST) : make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 2 * XR; ++k)
          if (p0 + k * NST < NP) stage(p0 + k * NST, t[k].x, t[k].y, make_float2(1.f, 1.f), 1.f);
      }
    } else {
      // RMSNorm is linear in its scale: the splits of w * x are staged at once and the finished strip
      // values (lattice, kink and low-rank terms alike) are multiplied by 1/rms, so the sum of squares
      // stays off the staging path; its per-warp parts are summed after the staging barrier
      float ss = 0.f;
      {  // the first XR pairs of this thread: all inputs in one batch of loads, weights loaded before the wait
        float2 xv[XR];
#pragma unroll
        for (int k = 0; k < XR; ++k) xv[k] = (tid + k * NST < NP) ? load_x(tid + k * NST) : make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < XR; ++k) {
          const int p = tid + k * NST;
          if (p < NP) {
            ss = fmaf(xv[k].x, xv[k].x, fmaf(xv[k].y, xv[k].y, ss));
            stage(p, xv[k].x, xv[k].y, wpre[k], 1.f);
          }
        }
      }
      for (int p0 = tid + XR * NST; p0 < NP; p0 += XR * NST) {
#pragma unroll
        for (int k = 0; k < XR; ++k) {
          const int p = p0 + k * NST;
          if (p < NP) {
            const float2 xv = load_x(p), wv = load_w(p);
            ss = fmaf(xv.x, xv.x, fmaf(xv.y, xv.y, ss));
            stage(p, xv.x, xv.y, wv, 1.f);
          }
        }
      }
      if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 11, tr_now());
      ss = warp_sum(ss);
      if (lane == 0) red[1 + warp] = ss;
    }
    if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 12, tr_now());
    // pairs past the row end of the last unit read zero activations
    for (int p = NP + tid; p < P.GU * HX_UB; p += NST) {
      const int j = p & 63, r = j & 15;
      const uint32_t off = xs_chunk((p >> 6) * 4 + (r >> 2), tab_off) + (uint32_t)((j >> 4) * 32 + (r & 3) * 4);
      *reinterpret_cast<uint32_t*>(smem + off) = 0u;
      *reinterpret_cast<uint32_t*>(smem + off + 16) = 0u;
    }
    for (int i = tid; i < P.n_local * width; i += NST) lacc[i] = 0ull;
    if (tid == 0) redu[38] = 0u;  // strips this CTA finished (decode kernel)
    named_bar_sync(1, NST);             // table, splits and accumulator ready for the streaming warps
    named_bar_arrive(2, HX_THREADS);    // ... and released to the helper warps
    if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 3, tr_now());

    if (MEGA && tid == 0) reinterpret_cast<int*>(redu)[35] = J.mat[0].radius;  // every streaming warp has read the old value
    const int pos = reinterpret_cast<const int*>(redu)[34];
    if (streamer) {
    // ---- streaming warps --------------------------------------------------------------
    const uint32_t lane4x = (uint32_t)lane * 4u | reinterpret_cast<const volatile uint32_t*>(redu)[32];
    const uint32_t dep = reinterpret_cast<const volatile uint32_t*>(redu)[33];  // zero, read after the barrier
    // B operand: lane (g, q) supplies column g.  Columns 0/1 (hi/lo of group A) are nonzero only
    // on the k rows of lanes q = 0, 1, columns 2/3 (group B) only on those of q = 2, 3, columns
    // 4-7 are zero.  The 8 lanes with data read one conflict-free 128-byte chunk per load.
    const bool bld = gl < 4 && ((gl >> 1) == (q >> 1));
    const uint32_t boff = (uint32_t)(q * 32 + (gl & 1) * 16);
    uint4 bv[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
    int cur_s = ns, cur_m = nm, cur_c = nc;
    if (u1 > u0 + 1) step_next();
    int seg_s = cur_s;
    float acc[NMAT][2];
#pragma unroll
    for (int mm = 0; mm < NMAT; ++mm) acc[mm][0] = acc[mm][1] = 0.f;
    auto emit = [&](int s) {  // this warp's part of strip s into the CTA's accumulator
      unsigned long long* la = lacc + (size_t)(s - s_lo) * width;
#pragma unroll
      for (int mm = 0; mm < NMAT; ++mm) {
        const float vg = acc[mm][0] + __shfl_xor_sync(0xffffffffu, acc[mm][0], 1);
        const float vh = acc[mm][1] + __shfl_xor_sync(0xffffffffu, acc[mm][1], 1);
        if (q == 0) {
          atomicAdd(la + mm * 16 + gl, hx_fix(vg));
          atomicAdd(la + mm * 16 + gl + 8, hx_fix(vh));
        }
      }
    };
    for (int u = u0; u < u1; ++u) {
      if (cur_s != seg_s) {
        emit(seg_s);
        seg_s = cur_s;
#pragma unroll
        for (int mm = 0; mm < NMAT; ++mm) acc[mm][0] = acc[mm][1] = 0.f;
      }
      const bool more = u + 1 < u1;
      // (pa, pb and the cursor point at unit u + 1 here) the unit pf_ahead past it goes into L2, so
      // that its register loads, issued one unit ahead, find it there; lane (g, q) takes one 128-byte
      // line: row g (q < 2) or g + 8, half q & 1
      if (FULL && !TMA && P.pf_ahead > 0 && more && nc + P.pf_ahead < P.GU) {
        const uint8_t* rowp = ((q >> 1) ? pb : pa) - q * 16 + P.pf_ahead * HX_UB + (q & 1) * 128;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(rowp));
      }
      // this unit's kink entries (range known since the previous unit) go into flight
      const uint32_t ko0 = nko0, ko1 = nko1;
      uint2 ke0 = make_uint2(0u, 0u), ke1 = make_uint2(0u, 0u);
      if (ukink && ko0 + lane < ko1) {
        const int km = (NMAT == 2) ? cur_m : strip_info<NMAT>(P, cur_s).m0;
        const uint2* kent = reinterpret_cast<const uint2*>(mp.mat(km).unit_kinks) + ko0 + lane;
        ke0 = __ldg(kent);
        if (ko0 + 32u + lane < ko1) ke1 = __ldg(kent + 32);
      }
      // this unit's scales; the next unit's scales go into flight
      uint32_t swa[4], swb[4];
      const int ch0 = cur_c * 16;
      const uint32_t bstride = ch0 < 256 ? 256u : 128u;
      const uint32_t bbase = sbase + xs_chunk(ch0, tab_off) + dep + boff;  // absolute shared address
      float rg_sum = 0.f, rh_sum = 0.f;
      if constexpr (TMA) {
        if (more && ukink) load_scales();  // the next unit's kink range
        const int slot = (u - u0) & 1;
        const uint32_t sl = slot0 + (uint32_t)(slot * HX_SLOT);
        if (!mbar_wait_bounded(bar0 + (uint32_t)(slot * 8), (ph >> slot) & 1u)) {
          if (MEGA && lane == 0 && mp.abort()) atomicExch(mp.abort(), 1u);
          break;  // a copy that never landed: the flag is raised, the strip results are void
        }
        ph ^= 1u << slot;
        const uint4 x = lds_u4(sl + 4096u + (uint32_t)(gl * 16)), y = lds_u4(sl + 4096u + (uint32_t)((gl + 8) * 16));
        swa[0] = x.x, swa[1] = x.y, swa[2] = x.z, swa[3] = x.w;
        swb[0] = y.x, swb[1] = y.y, swb[2] = y.z, swb[3] = y.w;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t cs = sl + (uint32_t)(s * 1024 + gl * 64 + q * 16);
          const uint4 ca = lds_u4(cs), cb = lds_u4(cs + 512u);
          float rg, rh;
          segment_mma(ca, cb, bbase + (uint32_t)s * 4u * bstride, bstride, bld, bv, lane4x, rg, rh);
          rg_sum = fmaf(h2f((uint16_t)(swa[s] >> sh)), rg, rg_sum);
          rh_sum = fmaf(h2f((uint16_t)(swb[s] >> sh)), rh, rh_sum);
        }
        // every lane's reads of the slot have been consumed by its MMAs: refill it two units ahead
        __syncwarp();
        if (u + 2 < u1 && lane == 0) {
          issue(slot);
          issue_next();
        }
      } else {
#pragma unroll
        for (int s = 0; s < 4; ++s) swa[s] = sa[s], swb[s] = sb[s];
        if (more) load_scales();
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          float rg, rh;
          segment_mma(cw[s][0], cw[s][1], bbase + (uint32_t)s * 4u * bstride, bstride, bld, bv, lane4x, rg, rh);
          if (more) load_codes(s);  // refill this segment's registers with the next unit
          rg_sum = fmaf(h2f((uint16_t)(swa[s] >> sh)), rg, rg_sum);
          rh_sum = fmaf(h2f((uint16_t)(swb[s] >> sh)), rh, rh_sum);
        }
      }
      if (ukink) {
        // the unit's kinks, sorted by row: a segmented scan per row, one writer per row
        auto kink_set = [&](uint2 e, bool valid) {
          const int col = (int)(e.x & 0xffffu), row = (int)(e.x >> 16) & 15;
          const bool ok = valid && col < C;
          float v = 0.f;
          if (ok) {
            const float2 xp = xs_pair(col >> 1);
            v = __uint_as_float(e.y) * ((col & 1) ? xp.y : xp.x);
          }
          if (valid && !ok) raise_flag(GSDLQ_FLAG_BAD_KINK);
          const int key = valid ? row : 64 + lane;
#pragma unroll
          for (int d = 1; d < 32; d <<= 1) {
            const float vu = __shfl_up_sync(0xffffffffu, v, d);
            const int ku = __shfl_up_sync(0xffffffffu, key, d);
            if (lane >= d && ku == key) v += vu;
          }
          const int kn = __shfl_down_sync(0xffffffffu, key, 1);
          if (valid && (lane == 31 || kn != key)) s_ks[row] += v;
          __syncwarp();
        };
        const uint32_t n = ko1 - ko0;
        if (n > 0u) {
          kink_set(ke0, lane < n);
          if (n > 32u) kink_set(ke1, lane + 32u < n);
          if (n > 64u) {  // rare: units with more than 64 kinks load the rest here
            const int km = (NMAT == 2) ? cur_m : strip_info<NMAT>(P, cur_s).m0;
            const uint2* kent = reinterpret_cast<const uint2*>(mp.mat(km).unit_kinks) + ko0;
            for (uint32_t b0 = 64u; b0 < n; b0 += 32u) {
              const bool valid = b0 + lane < n;
              kink_set(valid ? __ldg(kent + b0 + lane) : make_uint2(0u, 0u), valid);
            }
          }
          if (q == 0) {
            rg_sum += s_ks[gl];
            rh_sum += s_ks[gl + 8];
          }
          __syncwarp();
          if (lane < 16) s_ks[lane] = 0.f;
          __syncwarp();
        }
      }
      if (NMAT == 1 || cur_m == 0) {
        acc[0][0] += rg_sum;
        acc[0][1] += rh_sum;
      } else {
        acc[NMAT - 1][0] += rg_sum;
        acc[NMAT - 1][1] += rh_sum;
      }
      cur_s = ns, cur_m = nm, cur_c = nc;
      if (u + 2 < u1) step_next();
      if (tid == 0 && u == u0) GSDLQ_TR_SET(HX_SLOT_NOW, 13, tr_now());
    }
    if (lane == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 16 + warp, tr_now());
    if (TMA && MEGA && lane == 0) *ph_word = ph;  // the slots' parities carry over to the next phase
    if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 4, tr_now());
    if (lane == 0) GSDLQ_TR_MAX(HX_SLOT_NOW, 5);
    if (u1 > u0) emit(seg_s);
      }
  }

  // ---- finish this CTA's strips ------------------------------------------------------------
  // After one barrier every warp and helper term is in the accumulator.  Warp w takes strips
  // s_lo + w, s_lo + w + 16, ...: a strip inside this CTA's range is finished from the
  // accumulator; one shared with other CTAs adds its part to the strip's counted global words
  // (HX_SH_ONE), and the CTA that completes them finishes it and leaves them at zero.
  {
    // (the operands of this warp's first strip's epilogue are loaded before the barrier)
    const int pos = reinterpret_cast<const volatile int*>(redu)[34];
    StripPre sp0;
    if (s_lo + warp <= s_hi) sp0 = strip_pre<EPI>(P, strip_info<NMAT>(P, s_lo + warp), lane, pos);
    __syncthreads();
    if (tid == 0) GSDLQ_TR_SET(HX_SLOT_NOW, 6, tr_now());
    // the scale of the finished strip values: 1/rms of a normed input (the staging threads' sums of
    // squares are in the reduction words since the staging barrier), else 1
    float v_scale = 1.f;
    if (mp.input_mode() != GSDLQ_IN_PLAIN) {
      float tot = 0.f;
      for (int k = 0; k < HX_STREAM; ++k) tot += red[1 + k];
      v_scale = 1.0f / sqrtf(tot / (float)C + J.eps);  // gsd_lq_cpu_engine.c:78
    }
    unsigned nfin = 0u;
    // tensor parallelism: finished strips are posted to the peers here and summed after the loop
    const bool exch = EPI == GSDLQ_EPI_RESID && !MEGA && P.ex_on;
    const unsigned ex_k = exch ? redu[41] : 0u;
    unsigned ex_mask = 0u;  // loop iterations of this warp whose strip it posted
    int iter = -1;
    for (int s = s_lo + warp; s <= s_hi; s += HX_WARPS) {
      ++iter;
      const long long first = (long long)s * P.UPS;
      const int cf = hx_cta_of(P.T, P.n_cta, first), cl = hx_cta_of(P.T, P.n_cta, first + P.UPS - 1);
      const StripInfo si = strip_info<NMAT>(P, s);
      const StripPre sp = s == s_lo + warp ? sp0 : strip_pre<EPI>(P, si, lane, pos);
      unsigned long long a = lane < width ? lacc[(size_t)(s - s_lo) * width + lane] : 0ull;
      if (cf != cl) {
        unsigned long long* g = mp.gacc() + (size_t)s * width + lane;
        const unsigned total = (unsigned)(cl - cf + 1);
        unsigned long long w = 0ull;
        if (lane < width) w = atomicAdd(g, a + HX_SH_ONE) + a + HX_SH_ONE;  // the word after this addition
        if (__shfl_sync(0xffffffffu, hx_sh_count(w), 0) != total) continue;  // another CTA completes it
        if (lane < width) {
          // the other CTAs' additions to this lane's word were issued with their word-0 additions:
          // wait (bounded) for any still in flight
          unsigned long long t0 = 0ull;
          for (int it = 0; hx_sh_count(w) < total; ++it) {
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(g) : "memory");
            unsigned long long t1;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
            if (it == 0) t0 = t1;
            if (t1 - t0 > 1000000000ull) {
              raise_flag(GSDLQ_FLAG_TIMEOUT);
              break;
            }
          }
          a = w - (unsigned long long)total * HX_SH_ONE;
          *g = 0ull;  // the workspace is zero again for its next launch
        }
      }
      if (exch) {
        // this rank's partial of the strip's rows into every other rank's slots (value | call << 32);
        // kept in the accumulator word for the sum below
        const float pv = hx_unfix(a) * v_scale;
        const int row = si.rbase + (lane & 15);
        if (lane < 16 && row < J.mat[0].rows) {
          const unsigned long long w = ll_pack(pv, ex_k);
          for (int r = 0; r < P.ex.world; ++r)
            if (r != P.ex.rank) st_vol_u64(ex_slot(P.ex, r, ex_k, P.ex.rank, row), w);
          reinterpret_cast<float*>(lacc + (size_t)(s - s_lo) * width + lane)[0] = pv;
        }
        ex_mask |= 1u << iter;
        ++nfin;
        continue;
      }
      finish_value<EPI, NMAT>(P, mp, si, hx_unfix(a) * v_scale, lane, pos, sp);
      ++nfin;
    }
    if (exch) {
      // y = ((resid + p_0) + p_1) + ... in rank order (the peers' partials from this rank's slots,
      // bounded waits), the same bits on every rank
      unsigned long long deadline = 0ull;
      bool gave_up = false;
      for (int i = 0; i < 32 && (ex_mask >> i) != 0u; ++i) {
        if (((ex_mask >> i) & 1u) == 0u) continue;
        const int s = s_lo + warp + i * HX_WARPS;
        const StripInfo si = strip_info<NMAT>(P, s);
        const int row = si.rbase + (lane & 15);
        float out = 0.f;
        // one lane waits for each peer's strip (a peer posts a strip's 16 rows together), then the
        // others read their rows
        if (lane == 0)
          for (int r = 0; r < P.ex.world; ++r)
            if (r != P.ex.rank) (void)ex_wait(P.ex, ex_k, r, si.rbase, deadline, gave_up);
        __syncwarp();
        if (lane < 16 && row < J.mat[0].rows) {
          const float own = reinterpret_cast<const float*>(lacc + (size_t)(s - s_lo) * width + lane)[0];
          out = __ldcg(J.resid + row);
          for (int r = 0; r < P.ex.world; ++r) out += r == P.ex.rank ? own : ex_wait(P.ex, ex_k, r, row, deadline, gave_up);
          J.y[0][row] = out;
        }
        // low-rank forwarding of the summed rows into the next launch (the whole warp: shuffles)
        if (J.fwd_acc != nullptr) fwd_apply(J, fwd_load(J, si.rbase, J.mat[0].rows, lane), si.rbase, J.mat[0].rows, out, lane);
      }
      // the last CTA to get here advances the exchange's call number for the next such launch
      __syncthreads();
      if (tid == 0) {
        unsigned* w = ex_words(P.ex);
        if (atomicAdd(w + 1, 1u) == gridDim.x - 1) {
          w[1] = 0u;
          w[0] = ex_k;
        }
      }
    }
    if (lane == 0) GSDLQ_TR_MAX(HX_SLOT_NOW, 7);
    if (MEGA) {
      // one release per CTA: its finished strips and 1 for the CTA (it has read its input)
      if (lane == 0 && nfin) atomicAdd(&redu[38], nfin);
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        red_add_release(mp.done(), redu[38] + 1u);
      }
    }
  }
}

// UK: launches whose matrices carry per-unit kink lists (the streaming warps apply the kinks)
template <int EPI, bool FULL, bool TMA, bool UK>
__global__ void __launch_bounds__(HX_THREADS, 1) hexmv_kernel(const __grid_constant__ HexmvParams P,
                                                              const __grid_constant__ HxMaps T) {
  extern __shared__ __align__(1024) uint8_t smem[];
  hexmv_body<EPI, FULL, false, TMA, HxPtrs, UK>(P, HxPtrs{P, T}, smem);
}

}  // namespace gsdlq

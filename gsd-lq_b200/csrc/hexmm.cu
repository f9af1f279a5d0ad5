// hexmm.cu -- the batched packed linear: B <= 128 tokens through one GSD-LQ matrix as a dequant-GEMM on
// the 5th-generation tensor cores (tcgen05, accumulators in tensor memory) -- the batch-B counterpart of
// gsd_cpu_lowrank_proj + gsd_cpu_hex2d_matvec (gsd_lq_cpu_engine.c:111-183) applied to each token, used
// for batched decode and for chunked prefill.
//
//   y[b][r] = sum_c W[r][c] x[b][c] + sum_{kinks of r} delta * x[b][col] + sum_j U[r][j] tmp[b][j],
//   W[r][2p + i] = xy[code(r, p)][i] * scale(r, p / 32),  tmp[b][j] = S[j] * (Vt[j] . x[b]).
//
// One call is three launches: hexmm_prep (y zeroed, per-token max|x|, the low-rank projections tmp and a
// transposed fp32 copy of the activations), hexmm_xs_sparse (the activations as fp16 hi / lo B tiles, and
// the kink and low-rank terms of every (token, row) added into y) and hexmm_kernel, the dense lattice part,
// added into y with fp32 atomics (so the summation order is not fixed).  hexmm_kernel is a programmatic
// dependent launch: its set-up runs while hexmm_xs_sparse does, and only its B-tile loads wait for it.
//
// hexmm_kernel.  A CTA owns a tile of 128 weight rows (the tensor memory's lanes) and a contiguous run of
// 64-column k-blocks (split-K over CTAs, so that every SM streams weights).  Eight decoder warps, an issuer
// warp and a loader warp, linked by mbarriers; per k-block i:
//   - decoder thread t (row t % 128, columns 32 (t / 128) .. + 31 of the block) takes its 16 code bytes and
//     the row's scale from a cp.async ring, looks every code up in its lane's copy of the 256-entry decode
//     table (conflict-free) and forms the fp16 hi and lo parts of W = (x, r1) * (scale, scale sqrt3/2) in
//     fp16 arithmetic (hi the rounded product, lo the rounded remainder of a fused multiply-add: about 22
//     significant bits together), stores both with tcgen05.st into its tensor-memory lane as the A operand
//     of stage i % SA and arrives on the stage's full barrier;
//   - the loader bulk-copies block i's B tile (token b as two K-major 128-byte-swizzled rows: 2b = fp16 hi,
//     2b + 1 = fp16 lo of x_b scaled by a power of two that puts max|x_b| in [2^14, 2^15)) into shared
//     stage i % SB once the MMAs that read that stage before have completed;
//   - the issuer waits for both, issues eight tcgen05.mma (W hi and W lo per 16-column k-step; M = 128,
//     N = 2 x tokens padded to 8; A from tensor memory, B by descriptor; fp32 accumulate in tensor memory)
//     and commits them to the stages' empty barriers.
// At the end the decoder warps read the accumulator lanes with tcgen05.ld, add each token's hi and lo
// columns, unscale and add them into y.
#include <atomic>
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "common.cuh"

namespace gsdlq {

constexpr int MM_ROWS = 128;      // weight rows per CTA (tensor-memory lanes)
constexpr int MM_KB = 64;         // columns per k-block: one scale group
constexpr int MM_THREADS = 256;   // two threads per weight row (its two 32-column halves of a block)
constexpr int MM_MAXB = GSDLQ_MATMUL_MAX_BATCH;  // tokens per call (N = 2 * 128 = 256, the largest MMA N)
// decode table, header and B stages by absolute shared-window address (the layout is described below)
constexpr uint32_t MM_TAB_ABS = 0x1000u, MM_HDR_ABS = MM_TAB_ABS - 1024u, MM_B_ABS = MM_TAB_ABS + 0x10000u;
constexpr float MM_WF = 1024.f;                // power-of-two factor on the decoded weights

// Per group of 8 tokens (warp w: token 8 blockIdx.x + w) and chunk of MM_PREP columns: the chunk's
// max|x_b| into amax[b] (as ordered bits) and its part of S[j] * (Vt[j] . x_b) into tmp[16 b + j]
// (gsd_cpu_lowrank_proj; fp32 atomics, so the summation order is not fixed).  Both start at zero.  The
// warp stages x_b's chunk in shared memory; lane 2j + h then forms the dot product of Vt[j] with its
// half h of the chunk from sixteen 16-byte loads issued together.
constexpr int MM_PREP = 256;
__global__ void __launch_bounds__(256) hexmm_prep(const float* __restrict__ x, int B, int C,
                                                  const uint16_t* __restrict__ Vt, const float* __restrict__ S, int k,
                                                  unsigned* __restrict__ amax_bits, float* __restrict__ tmp,
                                                  float* __restrict__ xT, int BP, float* __restrict__ y, size_t yn) {
  __shared__ __align__(16) float xs[8][MM_PREP];
  {  // y starts at zero: the sparse pass and the dense kernel both add into it
    const size_t nthr = (size_t)gridDim.x * gridDim.y * blockDim.x;
    size_t i = ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i < yn; i += nthr) y[i] = 0.f;
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, b = blockIdx.x * 8 + w;
  const bool live = b < B;
  const int c0 = blockIdx.y * MM_PREP;
  const int j = lane >> 1, h = lane & 1, cc = c0 + h * (MM_PREP / 2);
  // the Vt loads first: they do not depend on x
  uint4 vt[MM_PREP / 16];
#pragma unroll
  for (int i = 0; i < MM_PREP / 16; ++i)
    vt[i] = (live && j < k && cc + 8 * i + 8 <= C)
                ? __ldg(reinterpret_cast<const uint4*>(Vt + (size_t)j * C + cc + 8 * i))
                : make_uint4(0u, 0u, 0u, 0u);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MM_PREP / 32; ++i) {
    const int c = c0 + lane + 32 * i;
    const float v = (live && c < C) ? x[(size_t)b * C + c] : 0.f;
    xs[w][lane + 32 * i] = v;
    amax = fmaxf(amax, fabsf(v));
  }
  amax = warp_max(amax);
  if (live && lane == 0) atomicMax(amax_bits + b, __float_as_uint(amax));  // non-negative floats order as bits
  __syncwarp();
  if (live) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < MM_PREP / 16; ++i) {
      const uint32_t q[4] = {vt[i].x, vt[i].y, vt[i].z, vt[i].w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        acc = fmaf(h2f((uint16_t)(q[t] & 0xffffu)), xs[w][h * (MM_PREP / 2) + 8 * i + 2 * t], acc);
        acc = fmaf(h2f((uint16_t)(q[t] >> 16)), xs[w][h * (MM_PREP / 2) + 8 * i + 2 * t + 1], acc);
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (h == 0 && j < k) atomicAdd(tmp + (size_t)b * 16 + j, S[j] * acc);
  }
  // xT[c][8 blockIdx.x .. + 7] for the CTA's columns (zero past the batch): one 32-byte row piece each
  __syncthreads();
  const int c = c0 + threadIdx.x;
  if (threadIdx.x < MM_PREP && c < C) {
    float4* dst = reinterpret_cast<float4*>(xT + (size_t)c * BP + blockIdx.x * 8);
    dst[0] = make_float4(xs[0][threadIdx.x], xs[1][threadIdx.x], xs[2][threadIdx.x], xs[3][threadIdx.x]);
    dst[1] = make_float4(xs[4][threadIdx.x], xs[5][threadIdx.x], xs[6][threadIdx.x], xs[7][threadIdx.x]);
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

// ---- tcgen05 helpers (cta_group::1) -----------------------------------------------------------
// shared-memory matrix descriptor: K-major, 128-byte swizzle (8-row x 128-byte atoms, SBO 1024 B
// between atoms; LBO unused for swizzled K-major), descriptor version 1.  The start address of k-step
// kk inside a 64-column block is the atom base + 32 kk bytes.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
// byte offset of 16-byte chunk j (columns 8j .. 8j+7) of row r in a swizzled 64-column tile
__device__ __forceinline__ int sw128(int r, int j) { return (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4); }
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 16 consecutive 32-bit columns of this thread's tensor-memory lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
// decode-table entry: byte permute of the code word and lane * 4 into (code << 8) | lane * 4, loaded with
// MM_TAB_ABS as the immediate offset (the table is constant after the set-up barrier)
__device__ __forceinline__ uint32_t mm_lookup(uint32_t word, uint32_t lane4, uint32_t sel) {
  const uint32_t a = __byte_perm(word, lane4, sel);
  uint32_t r;
  asm("ld.shared.b32 %0, [%1+%2];" : "=r"(r) : "r"(a), "n"(MM_TAB_ABS));
  return r;
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);  // a in the low half
  return *reinterpret_cast<const uint32_t*>(&h);
}

constexpr int MM_CSTAGES = 6;                  // k-blocks of codes in flight per CTA (cp.async ring)
// Shared memory, by absolute shared-window address (the dynamic allocation starts at the system-reserved
// bytes B below MM_HDR_ABS; the kernel checks that B leaves the header room):
//   [MM_HDR_ABS, MM_TAB_ABS)           barriers, tensor-memory slot, token scales (1 KB)
//   [MM_TAB_ABS, MM_TAB_ABS + 64 KB)   decode table: 256 rows of 256 bytes, row c = code c's entry in 32
//                                      lane copies (128 bytes), then a free 128-byte half; the free halves
//                                      of rows 0-191 hold the code ring (6 stages), those of rows 192-239
//                                      the scales
//   [MM_TAB_ABS + 64 KB, ...)          B stages (1024-byte aligned: the swizzle atoms)
template <int NB>
constexpr int mm_btile() {  // one k-block of the B operand: 16 NB rows (token hi / lo) x 128 bytes
  return 16 * NB * 128;
}
// Tensor memory: the accumulator (N = 16 NB columns, from column 0, rounded up to 64), then SA A stages of
// 64 columns (32 columns of fp16 pairs for the hi parts of a block's 64 weights per row, 32 for the lo).
template <int NB>
constexpr int mm_acc_cols() {
  return (16 * NB + 63) / 64 * 64;
}
template <int NB>
constexpr int mm_astages() {  // A stages in tensor memory
  return mm_acc_cols<NB>() == 128 ? 2 : 3;
}
template <int NB>
constexpr int mm_bstages() {  // B stages in shared memory
  return NB <= 2 ? 6 : NB <= 4 ? 4 : NB <= 8 ? 2 : 3;
}
template <int NB>
constexpr int mm_tcols() {  // the allocation: a power of two >= 32
  return mm_acc_cols<NB>() + 64 * mm_astages<NB>() <= 256 ? 256 : 512;
}
template <int NB>
constexpr int mm_smem() {  // the dynamic allocation for B = 0
  return (int)MM_B_ABS + mm_bstages<NB>() * mm_btile<NB>();
}
template <int NB>
constexpr int mm_per_sm() {  // resident CTAs per SM: shared memory and the 512 tensor-memory columns
  return std::min(std::min(8, (227 * 1024) / (mm_smem<NB>() + 1024)), 512 / mm_tcols<NB>());
}
static_assert(mm_per_sm<1>() == 2 && mm_per_sm<4>() == 2 && mm_per_sm<8>() == 2 && mm_per_sm<16>() == 1,
              "CTAs per SM");
// The small-batch kernel (up to MM_SMALL_NB token groups): integer A (32 columns per stage, no lo part) and
// SC accumulator slots of N = 16 NB columns, one per k-block in flight (the scale is applied per block).
constexpr int MM_SMALL_NB = 4;
template <int NB>
constexpr int ms_acc_stages() {
  return NB <= 2 ? 4 : 2;
}
template <int NB>
constexpr int ms_slot() {  // accumulator columns per slot: N rounded up to 32
  return (16 * NB + 31) / 32 * 32;
}
template <int NB>
constexpr int ms_acol() {  // first A-stage column: after the accumulator slots
  return ms_slot<NB>() * ms_acc_stages<NB>();
}
constexpr int MS_ASTAGES = 3;
template <int NB>
constexpr int ms_tcols() {
  return ms_acol<NB>() + 32 * MS_ASTAGES <= 256 ? 256 : 512;
}
static_assert(ms_tcols<1>() == 256 && ms_tcols<2>() == 256 && ms_tcols<3>() == 256 && ms_tcols<4>() == 256,
              "two small-batch CTAs share an SM's 512 tensor-memory columns");
static_assert(mm_per_sm<MM_SMALL_NB>() <= 2, "the small-batch kernel's CTAs per SM fit 512 tensor-memory columns");
// ring slot of (stage, row, half): table row 32 stage + row / 4, free half, 32-byte pair of the row's
// halves (XOR 16 on odd row quads, so that the 8 lanes of a 16-byte load phase hit 8 bank groups)
__host__ __device__ constexpr uint32_t mm_ring(int st, int r, int h) {
  return MM_TAB_ABS + (uint32_t)(st * 32 + r / 4) * 256u + 128u +
         ((uint32_t)((r & 3) * 32 + h * 16) ^ (uint32_t)(((r >> 2) & 1) * 16));
}
// scale-ring slot of (stage, half, row): the 4-byte scale pair, rows of 32 in the free halves of 192 ..
__host__ __device__ constexpr uint32_t mm_scring(int st, int h, int r) {
  return MM_TAB_ABS + (uint32_t)(32 * MM_CSTAGES + st * 8 + h * 4 + r / 32) * 256u + 128u + (uint32_t)(r % 32) * 4u;
}
static_assert(32 * MM_CSTAGES + 8 * MM_CSTAGES <= 256, "the code and scale rings fit the table rows' free halves");

// The B operand of every k-block, made once per call: token b's row of the block as fp16 hi (row 2b) and
// lo (row 2b + 1) of x_b scaled by its power of two, in the swizzled layout of a 64-column tile, one
// contiguous block of mm_btile<NB>() bytes per k-block (tokens past the batch are zero).
// A2: the pair (x[2p], x[2p+1]) is written as (a, b) = (x[2p], x[2p]/2 + sqrt3/2 x[2p+1]), the activations
// the integer lattice coordinates (r0, r1) of a code multiply: r0 a + r1 b = x-coord x[2p] + y-coord x[2p+1]
// with (x-coord, y-coord) = (r0 + r1/2, r1 sqrt3/2) the code's point (the small-batch kernel's operands).
template <int NB, bool A2 = false>
__device__ void hexmm_xconv_block(const float* __restrict__ x, int B, int C, const unsigned* __restrict__ amax_bits,
                                  uint8_t* __restrict__ xs, int kb) {
  constexpr int BP = 8 * NB;
  uint8_t* blk = xs + (size_t)kb * mm_btile<NB>();
  for (int e = threadIdx.x; e < BP * 8; e += 256) {
    const int b = e >> 3, j = e & 7;
    float v[8];
    if (b < B) {
      const float f = hexmm_xscale(amax_bits[b]);
      const float4* xp = reinterpret_cast<const float4*>(x + (size_t)b * C + kb * MM_KB + 8 * j);
      const float4 u0 = xp[0], u1 = xp[1];
      v[0] = u0.x * f, v[1] = u0.y * f, v[2] = u0.z * f, v[3] = u0.w * f;
      v[4] = u1.x * f, v[5] = u1.y * f, v[6] = u1.z * f, v[7] = u1.w * f;
      if (A2) {
#pragma unroll
        for (int t = 0; t < 4; ++t) v[2 * t + 1] = fmaf(0.8660254037844386f, v[2 * t + 1], 0.5f * v[2 * t]);
      }
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = 0.f;
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const __half2 hh = __floats2half2_rn(v[2 * t], v[2 * t + 1]);
      hi[t] = *reinterpret_cast<const uint32_t*>(&hh);
      lo[t] = pack_h2(v[2 * t] - __low2float(hh), v[2 * t + 1] - __high2float(hh));
    }
    *reinterpret_cast<uint4*>(blk + sw128(2 * b, j)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(blk + sw128(2 * b + 1, j)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// A-operand helpers: tcgen05.mma with A in tensor memory, B by shared-memory descriptor
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
// 16 consecutive 32-bit columns of this thread's tensor-memory lane
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Decode-table entry of code i: fp16 x (= r0 + r1 / 2, exact) low, fp16 r1 high, from the caller's xy table,
// which must hold the A2 lattice points (x, r1 sqrt3/2) (checked, as the matvec checks it); codes past the
// last point decode to (0, 0).  The weights are x * scale and r1 * (scale * sqrt3/2).
__device__ __forceinline__ uint32_t mm_entry(const float* xy, int n_pts, int i) {
  if (i >= n_pts) return 0u;
  const float x = xy[2 * i], y = xy[2 * i + 1];
  const float r1 = rintf(y * 1.1547005383792515f);
  const float r0 = x - 0.5f * r1;
  if (r0 != rintf(r0) || (float)((double)r1 * 0.8660254037844386) != y || fabsf(r0) > 16.f || fabsf(r1) > 16.f) {
    raise_flag(GSDLQ_FLAG_BAD_TABLE);
    return 0u;
  }
  return pack_h2(x, r1);
}

// The kink and low-rank terms, added into y (zeroed by hexmm_prep; the dense kernel adds to it too).  One warp
// per weight row, lane = token b, b + 32, ... (up to four chunks of 32): the row's kinks are loaded 32 at
// a time and broadcast eight at a time, each adds delta * xT[col][b] (the activation loads of the eight
// kinks and every token chunk issued together); then U[row] . tmp[b] (gsd_cpu_hex2d_matvec's kink loop
// and gsd_cpu_lowrank_proj's second half, gsd_lq_cpu_engine.c:111-183).
__device__ void hexmm_sparse_rows(const float* __restrict__ xT, int BP, int B, int R, int C,
                                  const uint32_t* __restrict__ row_ptr, const uint16_t* __restrict__ kcols,
                                  const float* __restrict__ kdel, const uint16_t* __restrict__ U, int k,
                                  const float* __restrict__ tmp, float* __restrict__ y, int rb, float* tmp_s) {
  constexpr int TC = MM_MAXB / 32;  // token chunks
  // tmp_s: tmp[b][j] at 17 b + j, so that lane b's reads hit 32 banks
  if (k > 0) {
    for (int i = threadIdx.x; i < B * 16; i += blockDim.x) tmp_s[(i >> 4) * 17 + (i & 15)] = tmp[i];
    __syncthreads();
  }
  const int lane = threadIdx.x & 31, row = rb * 8 + (threadIdx.x >> 5);
  if (row >= R) return;
  const uint32_t e0 = row_ptr[row], e1 = row_ptr[row + 1];
  if (e0 == e1 && k == 0) return;  // nothing to add (Turbo rows)
  const int nch = (B + 31) / 32;
  float acc[TC];
#pragma unroll
  for (int t = 0; t < TC; ++t) acc[t] = 0.f;
  for (uint32_t e = e0; e < e1; e += 32) {
    const uint32_t my = e + lane;
    int col = my < e1 ? (int)kcols[my] : 0;
    float d = my < e1 ? kdel[my] : 0.f;
    if (col >= C) {  // past the row: the reference rejects the matrix
      raise_flag(GSDLQ_FLAG_BAD_KINK);
      col = 0;
      d = 0.f;
    }
    const int n = (int)min(32u, e1 - e);  // the kinks past the row's end have delta 0 and column 0
    for (int j0 = 0; j0 < n; j0 += 8) {
      int cj[8];
      float dv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cj[j] = __shfl_sync(0xffffffffu, col, j0 + j);
        dv[j] = __shfl_sync(0xffffffffu, d, j0 + j);
      }
#pragma unroll
      for (int t = 0; t < TC; ++t) {
        if (t < nch) {
          const int bb = min(32 * t + lane, BP - 1);
          float xv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = __ldg(xT + (size_t)cj[j] * BP + bb);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[t] = fmaf(dv[j], xv[j], acc[t]);
        }
      }
    }
  }
  float u[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) u[j] = j < k ? h2f(U[(size_t)row * k + j]) : 0.f;
#pragma unroll
  for (int t = 0; t < TC; ++t) {
    const int b = 32 * t + lane;
    if (t < nch && b < B) {
      float lrv = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < k) lrv = fmaf(u[j], tmp_s[b * 17 + j], lrv);
      atomicAdd(y + (size_t)b * R + row, acc[t] + lrv);
    }
  }
}

// The B tiles (CTAs 0 .. nkb - 1, one k-block each) and the sparse terms (the rest, 8 rows each) in one
// launch: both need only hexmm_prep's results.  Every CTA lets the dense kernel launch at once
// (programmatic dependent launch); that kernel waits for this one only before its first B-tile copy.
template <int NB, bool A2>
__global__ void __launch_bounds__(256) hexmm_xs_sparse(const float* __restrict__ x, int B, int C,
                                                       const unsigned* __restrict__ amax_bits,
                                                       uint8_t* __restrict__ xs, int nkb,
                                                       const float* __restrict__ xT, int R,
                                                       const uint32_t* __restrict__ row_ptr,
                                                       const uint16_t* __restrict__ kcols,
                                                       const float* __restrict__ kdel,
                                                       const uint16_t* __restrict__ U, int k,
                                                       const float* __restrict__ tmp, float* __restrict__ y) {
  __shared__ float tmp_s[MM_MAXB * 17];
  asm volatile("griddepcontrol.launch_dependents;");
  if ((int)blockIdx.x < nkb)
    hexmm_xconv_block<NB, A2>(x, B, C, amax_bits, xs, blockIdx.x);
  else
    hexmm_sparse_rows(xT, 8 * NB, B, R, C, row_ptr, kcols, kdel, U, k, tmp, y, blockIdx.x - nkb, tmp_s);
}

// NB: groups of 8 tokens (tokens padded to 8 NB with zero activations); N = 16 NB accumulator columns.
// Threads 0-255 decode (thread t: half t / 128 of weight row t % 128, written into tensor-memory lane t % 128
// by warp t / 32, whose lane quarter is warp % 4); warp 8 issues the MMAs, warp 9 bulk-copies the B tiles.
constexpr int MM_ALL = MM_THREADS + 64;
template <int NB>
__global__ void __launch_bounds__(MM_ALL) hexmm_kernel(const uint8_t* __restrict__ xs, int B,
                                                       const uint8_t* __restrict__ codes,
                                                       const uint16_t* __restrict__ scales,
                                                       const float* __restrict__ xy, int n_pts,
                                                       float* __restrict__ y, int R, int C, int nsplit,
                                                       const unsigned* __restrict__ amax_bits) {
  constexpr int N = 16 * NB, BP = 8 * NB, SA = mm_astages<NB>(), SB = mm_bstages<NB>();
  constexpr uint32_t TCOLS = (uint32_t)mm_tcols<NB>(), ACOL = (uint32_t)mm_acc_cols<NB>();
  constexpr int BTILE = mm_btile<NB>();
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t sbase = smem_u32(sm);
  if (sbase > MM_HDR_ABS) {  // the layout's assumption on the reserved bytes
    if (threadIdx.x == 0) raise_flag(GSDLQ_FLAG_UNSUPPORTED);
    return;
  }
  // header: barriers afull[SA] | aempty[SA] | bfull[SB] | bempty[SB] (8 bytes each, 64 apart), the
  // tensor-memory slot, token scales
  uint8_t* hdr = sm + (MM_HDR_ABS - sbase);
  const uint32_t afull = MM_HDR_ABS, aempty = MM_HDR_ABS + 64, bfull = MM_HDR_ABS + 128, bempty = MM_HDR_ABS + 192;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(hdr + 256);
  float* inv_xsc = reinterpret_cast<float*>(hdr + 512);            // [MM_MAXB]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * MM_ROWS, split = blockIdx.y;
  const int NP = C / 2, G = C / 64, nkb = C / MM_KB;
  const int kb0 = (int)((long long)nkb * split / nsplit), kb1 = (int)((long long)nkb * (split + 1) / nsplit);
  const int nk = kb1 - kb0;
  // scale pairs by cp.async when every row's scales start on a 4-byte boundary
  const bool sc_async = (G % 2 == 0) && ((reinterpret_cast<uintptr_t>(scales) & 3u) == 0);
  const int lr = tid & (MM_ROWS - 1), half = (tid >> 7) & 1;
  const int row = r0 + lr;
  const bool rok = tid < MM_THREADS && row < R;
  const uint8_t* cp = codes + (size_t)(rok ? row : 0) * NP + half * 16;
  const uint16_t* scp = scales + (size_t)(rok ? row : 0) * G;
  // decoder: this thread's 16 code bytes (and its row's pair of scales) of k-block kb0 + i into ring
  // stage i % MM_CSTAGES (one group per block, empty past the run, so that the group count stays uniform)
  auto fetch = [&](int i) {
    if (i < nk && rok) {
      const int st = i % MM_CSTAGES;
      cp_async_16(sm + (mm_ring(st, lr, half) - sbase), cp + (kb0 + i) * 32);
      if (sc_async) cp_async_4(sm + (mm_scring(st, half, lr) - sbase), scp + ((kb0 + i) & ~1));
    }
    cp_async_commit();
  };
  if (tid < MM_THREADS) {
#pragma unroll
    for (int i = 0; i < MM_CSTAGES - 1; ++i) fetch(i);
    const uint32_t ent = mm_entry(xy, n_pts, tid);
#pragma unroll 8
    for (int i = 0; i < 32; ++i) st_shared_u32(MM_TAB_ABS + (uint32_t)tid * 256u + (uint32_t)((i + tid) & 31) * 4u, ent);
    if (tid < BP) inv_xsc[tid] = tid < B ? 1.0f / (hexmm_xscale(amax_bits[tid]) * MM_WF) : 0.f;
  }
  if (tid == 0) {
#pragma unroll
    for (int q = 0; q < SA; ++q) {
      mbar_init(afull + 8u * q, (uint32_t)MM_THREADS);
      mbar_init(aempty + 8u * q, 1u);
    }
#pragma unroll
    for (int q = 0; q < SB; ++q) {
      mbar_init(bfull + 8u * q, 1u);
      mbar_init(bempty + 8u * q, 1u);
    }
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);
#ifdef GSDLQ_TRACE
  const bool trc = blockIdx.y == 0;
#endif

  if (warp == MM_THREADS / 32 + 1) {
    // ---- B loader: block j's tile into stage j % SB once the MMAs of block j - SB have completed ----
    if (lane == 0) {
      // the tiles are written by the launch before this one (programmatic dependent launch): wait for it
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int q = 0;
      uint32_t pe = 1u;  // parity of the empty phase to wait for (none on the first pass)
      for (int j = 0; j < nk; ++j) {
        if (j >= SB) mbar_wait_bounded(bempty + 8u * q, pe);
        mbar_arrive_expect_tx(bfull + 8u * q, (uint32_t)BTILE);
        bulk_g2s(MM_B_ABS + q * BTILE, xs + (size_t)(kb0 + j) * BTILE, (uint32_t)BTILE, bfull + 8u * q);
        if (++q == SB) q = 0, pe ^= 1u;
      }
    }
  } else if (warp == MM_THREADS / 32) {
    // ---- issuer ----
    if (lane == 0) {
#ifdef GSDLQ_TRACE
      if (trc) GSDLQ_TR_SET(0u, 21, tr_now());
#endif
      // instruction descriptor: D fp32, A and B fp16, both K-major, N, M = 128
      const uint32_t idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(MM_ROWS >> 4) << 24);
      int qa = 0, qb = 0;
      uint32_t pa = 0u, pb = 0u;  // stage indices and their phase parities
      for (int i = 0; i < nk; ++i) {
        mbar_wait_bounded(afull + 8u * qa, pa);  // the decoders' A parts of block i
        mbar_wait_bounded(bfull + 8u * qb, pb);  // its B tile
        tc_fence_after();
#ifdef GSDLQ_TRACE
        if (trc && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 5, tr_now());
#endif
#pragma unroll
        for (int kk = 0; kk < MM_KB / 16; ++kk) {
          const uint64_t bd = umma_desc(MM_B_ABS + qb * BTILE + kk * 32);
          const uint32_t aa = tmem + ACOL + 64u * (uint32_t)qa + 8u * (uint32_t)kk;
          umma_f16_ts(tmem, aa, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          umma_f16_ts(tmem, aa + 32u, bd, idesc, 1u);
        }
        umma_commit(aempty + 8u * qa);  // arrive when every MMA issued so far has completed
        umma_commit(bempty + 8u * qb);
        if (++qa == SA) qa = 0, pa ^= 1u;
        if (++qb == SB) qb = 0, pb ^= 1u;
#ifdef GSDLQ_TRACE
        if (trc && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 6, tr_now());
#endif
      }
    }
  } else {
    // ---- decoders ----
    const uint32_t lane4 = (uint32_t)lane * 4u;
    const uint32_t my_lane = (uint32_t)((warp & 3) * 32) << 16;  // this warp's tensor-memory lane quarter
    uint32_t cmax = 0u;  // byte-wise maximum of the codes seen (the bad-code check)
    bool bad_scale = false;
    int q = 0;
    uint32_t pe = 1u;  // A stage and the parity of its empty phase to wait for (none on the first pass)
    for (int i = 0; i < nk; ++i) {
      const int kb = kb0 + i, st = i % MM_CSTAGES;
#ifdef GSDLQ_TRACE
      if (trc && tid == 0 && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2), tr_now());
#endif
      fetch(i + MM_CSTAGES - 1);          // codes of the block MM_CSTAGES - 1 ahead
      cp_async_wait<MM_CSTAGES - 1>();    // this thread's codes of block i have landed
#ifdef GSDLQ_TRACE
      if (trc && tid == 0 && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 1, tr_now());
#endif
      uint32_t scw;
      if (sc_async) {
        scw = ld_shared_u32(mm_scring(st, half, lr));
        scw = (kb & 1) ? scw >> 16 : scw & 0xffffu;
      } else {
        scw = rok ? scp[kb] : 0u;
      }
      // W = (x, r1) * (scale, scale sqrt3/2) in fp16 hi + lo parts, computed in fp16 arithmetic: hi is the
      // rounded product, lo the rounded remainder (one fused multiply-add each: exact before rounding), and
      // the y part's factor scale sqrt3/2 (not an fp16 number) enters as its own fp16 hi + lo pair
      // The weights carry the factor MM_WF = 2^10 (removed in the epilogue), which keeps the lo parts of
      // weights above 2^-12 normal; |lattice x| <= 12, so scales up to 4.8 stay below fp16's 65504.
      const float s = h2f((uint16_t)scw) * MM_WF, sy = s * 0.8660254037844386f;
      if (!(fabsf(s) <= 5.0f * MM_WF)) bad_scale = true;
      const __half syh = __float2half_rn(sy);
      const __half syl = __float2half_rn(sy - __half2float(syh));
      const __half2 sc2 = __halves2half2(__float2half_rn(s), syh);
      const __half2 sl2 = __halves2half2(__float2half_rn(0.f), syl);
      const uint4 cw = *reinterpret_cast<const uint4*>(sm + (mm_ring(st, lr, half) - sbase));
      const uint32_t cv[4] = {cw.x, cw.y, cw.z, cw.w};
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        cmax = __vmaxu4(cmax, cv[jj]);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          // one byte permute makes (code << 8) | lane * 4, the entry of this lane's table copy
          const uint32_t ent = mm_lookup(cv[jj], lane4, 0x6604u | (uint32_t)(p << 4));
          const __half2 v = *reinterpret_cast<const __half2*>(&ent);
          const __half2 h = __hmul2(v, sc2);
          __half2 l = __hfma2(v, sc2, __hneg2(h));
          l = __hfma2(v, sl2, l);
          hi[4 * jj + p] = *reinterpret_cast<const uint32_t*>(&h);
          lo[4 * jj + p] = *reinterpret_cast<const uint32_t*>(&l);
        }
      }
#ifdef GSDLQ_TRACE
      if (trc && tid == 0 && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 2, (unsigned long long)hi[15] * 0ull + tr_now());
#endif
      // stage q is free once the MMAs of block i - SA have completed
      if (i >= SA) mbar_wait_bounded(aempty + 8u * q, pe);
      tc_fence_after();
#ifdef GSDLQ_TRACE
      if (trc && tid == 0 && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 3, tr_now());
#endif
      __syncwarp();
      const uint32_t acol = tmem + my_lane + ACOL + 64u * (uint32_t)q + 16u * (uint32_t)half;
      tmem_st16(acol, hi);
      tmem_st16(acol + 32u, lo);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive1(afull + 8u * q);
      if (++q == SA) q = 0, pe ^= 1u;
#ifdef GSDLQ_TRACE
      if (trc && tid == 0 && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 4, tr_now());
#endif
    }
    cp_async_wait<0>();
    {  // a code byte >= n_pts has no point in the table
      const uint32_t mx = max(max(cmax & 0xffu, (cmax >> 8) & 0xffu), max((cmax >> 16) & 0xffu, cmax >> 24));
      if (rok && (int)mx >= n_pts) raise_flag(GSDLQ_FLAG_BAD_CODE);
      if (rok && bad_scale) raise_flag(GSDLQ_FLAG_RANGE);
    }
    // ---- the run's partial sums: column pair (2b, 2b + 1) = token b's hi and lo parts; warp w reads the
    // lanes of its quarter, the 16-column groups cb with cb % 2 == w / 4 ----
    mbar_wait_bounded(aempty + 8u * ((nk - 1) % SA), (uint32_t)(((nk - 1) / SA) & 1));
    tc_fence_after();
    __syncwarp();
#ifdef GSDLQ_TRACE
    if (trc && tid == 0) GSDLQ_TR_SET(0u, 25, tr_now());
#endif
    const int erow = r0 + (warp & 3) * 32 + lane;
#pragma unroll 1
    for (int cb = warp >> 2; cb < N / 16; cb += 2) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(cb * 16), v);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int b = cb * 8 + t;
        if (erow < R && b < B)
          atomicAdd(y + (size_t)b * R + erow, (__uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1])) * inv_xsc[b]);  // includes 1 / MM_WF
      }
    }
#ifdef GSDLQ_TRACE
    if (trc && tid == 0) {
      GSDLQ_TR_SET(0u, 26, tr_now());
      GSDLQ_TR_SET(0u, 28, (unsigned long long)nk);
    }
#endif
  }
  // ---- release the tensor memory (every warp's tensor-memory accesses are complete) ----
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TCOLS);
  }
}

// Decode-table entry of the small-batch kernel: the code's integer lattice coordinates (r0, r1) as fp16
// (exact), from the caller's xy table (checked to be the A2 lattice, as mm_entry does).
__device__ __forceinline__ uint32_t ms_entry(const float* xy, int n_pts, int i) {
  if (i >= n_pts) return 0u;
  const float x = xy[2 * i], y = xy[2 * i + 1];
  const float r1 = rintf(y * 1.1547005383792515f);
  const float r0 = x - 0.5f * r1;
  if (r0 != rintf(r0) || (float)((double)r1 * 0.8660254037844386) != y || fabsf(r0) > 16.f || fabsf(r1) > 16.f) {
    raise_flag(GSDLQ_FLAG_BAD_TABLE);
    return 0u;
  }
  return pack_h2(r0, r1);
}

// The small-batch dense kernel (up to 8 MM_SMALL_NB tokens).  The weights enter the tensor cores as their
// integer lattice coordinates (exact in fp16, no lo part, no scale) against the A2-transformed activations,
// and every 64-column k-block (one scale group) accumulates into its own tensor-memory slot: decoder
// thread t reads its row's slot of block i - (SC - 1) with tcgen05.ld and adds scale x (hi + lo) of each
// token in its half of the slot to registers, then frees the slot.  Per code the decoders do one byte
// permute and one shared load.  Roles, rings, the table layout and the loader are those of hexmm_kernel.
template <int NB>
__global__ void __launch_bounds__(MM_ALL) hexmm_small_kernel(const uint8_t* __restrict__ xs, int B,
                                                             const uint8_t* __restrict__ codes,
                                                             const uint16_t* __restrict__ scales,
                                                             const float* __restrict__ xy, int n_pts,
                                                             float* __restrict__ y, int R, int C, int nsplit,
                                                             const unsigned* __restrict__ amax_bits) {
  constexpr int N = 16 * NB, BP = 8 * NB, SA = MS_ASTAGES, SB = mm_bstages<NB>(), SC = ms_acc_stages<NB>();
  constexpr int HT = 4 * NB;  // tokens in a thread's half of a slot
  constexpr uint32_t TCOLS = (uint32_t)ms_tcols<NB>(), ACOL = (uint32_t)ms_acol<NB>(), SLOT = (uint32_t)ms_slot<NB>();
  constexpr int BTILE = mm_btile<NB>();
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t sbase = smem_u32(sm);
  if (sbase > MM_HDR_ABS) {  // the layout's assumption on the reserved bytes
    if (threadIdx.x == 0) raise_flag(GSDLQ_FLAG_UNSUPPORTED);
    return;
  }
  // header: afull[SA] | aempty[SA] | bfull[SB] | bempty[SB] | cfull[SC] | cfree[SC] (8 bytes each), the
  // tensor-memory slot, token scales
  uint8_t* hdr = sm + (MM_HDR_ABS - sbase);
  const uint32_t afull = MM_HDR_ABS, aempty = MM_HDR_ABS + 32, bfull = MM_HDR_ABS + 64, bempty = MM_HDR_ABS + 128;
  const uint32_t cfull = MM_HDR_ABS + 192, cfree = MM_HDR_ABS + 224;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(hdr + 256);
  float* inv_xsc = reinterpret_cast<float*>(hdr + 512);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * MM_ROWS, split = blockIdx.y;
  const int NP = C / 2, G = C / 64, nkb = C / MM_KB;
  const int kb0 = (int)((long long)nkb * split / nsplit), kb1 = (int)((long long)nkb * (split + 1) / nsplit);
  const int nk = kb1 - kb0;
  const bool sc_async = (G % 2 == 0) && ((reinterpret_cast<uintptr_t>(scales) & 3u) == 0);
  const int lr = tid & (MM_ROWS - 1), half = (tid >> 7) & 1;
  const int row = r0 + lr;
  const bool rok = tid < MM_THREADS && row < R;
  const uint8_t* cp = codes + (size_t)(rok ? row : 0) * NP + half * 16;
  const uint16_t* scp = scales + (size_t)(rok ? row : 0) * G;
  auto fetch = [&](int i) {
    if (i < nk && rok) {
      const int st = i % MM_CSTAGES;
      cp_async_16(sm + (mm_ring(st, lr, half) - sbase), cp + (kb0 + i) * 32);
      if (sc_async) cp_async_4(sm + (mm_scring(st, half, lr) - sbase), scp + ((kb0 + i) & ~1));
    }
    cp_async_commit();
  };
  if (tid < MM_THREADS) {
#pragma unroll
    for (int i = 0; i < MM_CSTAGES - 1; ++i) fetch(i);
    const uint32_t ent = ms_entry(xy, n_pts, tid);
#pragma unroll 8
    for (int i = 0; i < 32; ++i) st_shared_u32(MM_TAB_ABS + (uint32_t)tid * 256u + (uint32_t)((i + tid) & 31) * 4u, ent);
    if (tid < BP) inv_xsc[tid] = tid < B ? 1.0f / hexmm_xscale(amax_bits[tid]) : 0.f;
  }
  if (tid == 0) {
#pragma unroll
    for (int q = 0; q < SA; ++q) {
      mbar_init(afull + 8u * q, (uint32_t)MM_THREADS);
      mbar_init(aempty + 8u * q, 1u);
    }
#pragma unroll
    for (int q = 0; q < SB; ++q) {
      mbar_init(bfull + 8u * q, 1u);
      mbar_init(bempty + 8u * q, 1u);
    }
#pragma unroll
    for (int q = 0; q < SC; ++q) {
      mbar_init(cfull + 8u * q, 1u);
      mbar_init(cfree + 8u * q, (uint32_t)MM_THREADS);
    }
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);

  if (warp == MM_THREADS / 32 + 1) {
    // ---- B loader (as in hexmm_kernel) ----
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int q = 0;
      uint32_t pe = 1u;
      for (int j = 0; j < nk; ++j) {
        if (j >= SB) mbar_wait_bounded(bempty + 8u * q, pe);
        mbar_arrive_expect_tx(bfull + 8u * q, (uint32_t)BTILE);
        bulk_g2s(MM_B_ABS + q * BTILE, xs + (size_t)(kb0 + j) * BTILE, (uint32_t)BTILE, bfull + 8u * q);
        if (++q == SB) q = 0, pe ^= 1u;
      }
    }
  } else if (warp == MM_THREADS / 32) {
    // ---- issuer: block i's four MMAs into accumulator slot i % SC (which the decoders have freed) ----
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(MM_ROWS >> 4) << 24);
      int qa = 0, qb = 0, qc = 0;
      uint32_t pa = 0u, pb = 0u, pc = 1u;
#ifdef GSDLQ_TRACE
      const bool trc = blockIdx.y == 0;
      if (trc) GSDLQ_TR_SET(0u, 21, tr_now());
#endif
      for (int i = 0; i < nk; ++i) {
        mbar_wait_bounded(afull + 8u * qa, pa);
        mbar_wait_bounded(bfull + 8u * qb, pb);
        if (i >= SC) mbar_wait_bounded(cfree + 8u * qc, pc);
        tc_fence_after();
#ifdef GSDLQ_TRACE
        if (trc && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 5, tr_now());
#endif
#pragma unroll
        for (int kk = 0; kk < MM_KB / 16; ++kk) {
          const uint64_t bd = umma_desc(MM_B_ABS + qb * BTILE + kk * 32);
          umma_f16_ts(tmem + SLOT * (uint32_t)qc, tmem + ACOL + 32u * (uint32_t)qa + 8u * (uint32_t)kk, bd, idesc,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(aempty + 8u * qa);
        umma_commit(bempty + 8u * qb);
        umma_commit(cfull + 8u * qc);
#ifdef GSDLQ_TRACE
        if (trc && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 6, tr_now());
#endif
        if (++qa == SA) qa = 0, pa ^= 1u;
        if (++qb == SB) qb = 0, pb ^= 1u;
        if (++qc == SC) qc = 0, pc ^= 1u;
      }
    }
  } else {
    // ---- decoders ----
    const uint32_t lane4 = (uint32_t)lane * 4u;
    const uint32_t my_lane = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t cmax = 0u;
    float yacc[HT];
#pragma unroll
    for (int t = 0; t < HT; ++t) yacc[t] = 0.f;
    float shist[SC];  // the scales of the blocks whose slots are still to be read, oldest first
#pragma unroll
    for (int t = 0; t < SC; ++t) shist[t] = 0.f;
    int qa = 0, qc = 0;
    uint32_t pea = 1u, pfc = 0u;
    // block j's slot: wait for its MMAs, add scale x (hi + lo) per token of this thread's half, free it
    auto drain = [&](float sj) {
      mbar_wait_bounded(cfull + 8u * qc, pfc);
      tc_fence_after();
      __syncwarp();
      // the slot's N columns in aligned 16-column loads (8 tokens each); this thread keeps its half's tokens
      uint32_t v[16];
#pragma unroll
      for (int c = 0; c < N / 16; ++c) {
        tmem_ld16(tmem + my_lane + SLOT * (uint32_t)qc + (uint32_t)(16 * c), v);
        if (half == 0) {
#pragma unroll
          for (int t = 0; t < 8; ++t)
            if (8 * c + t < HT)
              yacc[8 * c + t] = fmaf(sj, __uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1]), yacc[8 * c + t]);
        } else {
#pragma unroll
          for (int t = 0; t < 8; ++t)
            if (8 * c + t >= HT && 8 * c + t < 2 * HT)
              yacc[8 * c + t - HT] =
                  fmaf(sj, __uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1]), yacc[8 * c + t - HT]);
        }
      }
      tc_fence_before();
      mbar_arrive1(cfree + 8u * qc);
      if (++qc == SC) qc = 0, pfc ^= 1u;
    };
#ifdef GSDLQ_TRACE
    const bool trd = blockIdx.y == 0 && tid == 0;
#endif
    for (int i = 0; i < nk; ++i) {
      const int kb = kb0 + i, st = i % MM_CSTAGES;
#ifdef GSDLQ_TRACE
      if (trd && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2), tr_now());
#endif
      fetch(i + MM_CSTAGES - 1);
      cp_async_wait<MM_CSTAGES - 1>();
#ifdef GSDLQ_TRACE
      if (trd && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 1, tr_now());
#endif
      uint32_t scw;
      if (sc_async) {
        scw = ld_shared_u32(mm_scring(st, half, lr));
        scw = (kb & 1) ? scw >> 16 : scw & 0xffffu;
      } else {
        scw = rok ? scp[kb] : 0u;
      }
      const uint4 cw = *reinterpret_cast<const uint4*>(sm + (mm_ring(st, lr, half) - sbase));
      const uint32_t cv[4] = {cw.x, cw.y, cw.z, cw.w};
      uint32_t a[16];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        cmax = __vmaxu4(cmax, cv[jj]);
#pragma unroll
        for (int p = 0; p < 4; ++p) a[4 * jj + p] = mm_lookup(cv[jj], lane4, 0x6604u | (uint32_t)(p << 4));
      }
#ifdef GSDLQ_TRACE
      if (trd && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 2, (unsigned long long)a[15] * 0ull + tr_now());
#endif
      if (i >= SA) mbar_wait_bounded(aempty + 8u * qa, pea);
      tc_fence_after();
#ifdef GSDLQ_TRACE
      if (trd && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 3, tr_now());
#endif
      __syncwarp();
      tmem_st16(tmem + my_lane + ACOL + 32u * (uint32_t)qa + 16u * (uint32_t)half, a);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive1(afull + 8u * qa);
#ifdef GSDLQ_TRACE
      if (trd && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 7 * (i - 2) + 4, tr_now());
#endif
      if (++qa == SA) qa = 0, pea ^= 1u;
      // the scale of block i joins the history; the slot of block i - (SC - 1) is read
#pragma unroll
      for (int t = 0; t < SC - 1; ++t) shist[t] = shist[t + 1];
      shist[SC - 1] = h2f((uint16_t)scw);
      if (i >= SC - 1) drain(shist[0]);
#ifdef GSDLQ_TRACE
      if (trd && i >= 2 && i < 5) GSDLQ_TR_SET(0u, 22 + (i - 2), tr_now());
#endif
    }
#ifdef GSDLQ_TRACE
    if (trd) GSDLQ_TR_SET(0u, 25, tr_now());
    if (trd) GSDLQ_TR_SET(0u, 28, (unsigned long long)nk);
#endif
    // the last SC - 1 blocks' slots (fewer when the run is shorter)
    for (int t = 0; t < SC - 1; ++t) {
      if (nk - (SC - 1) + t >= 0) {
        float sj = 0.f;
#pragma unroll
        for (int u = 0; u < SC; ++u)
          if (u == t + 1) sj = shist[u];
        drain(sj);
      }
    }
    cp_async_wait<0>();
    {
      const uint32_t mx = max(max(cmax & 0xffu, (cmax >> 8) & 0xffu), max((cmax >> 16) & 0xffu, cmax >> 24));
      if (rok && (int)mx >= n_pts) raise_flag(GSDLQ_FLAG_BAD_CODE);
    }
    if (row < R && tid < MM_THREADS) {
#pragma unroll
      for (int t = 0; t < HT; ++t) {
        const int b = half * HT + t;
        if (b < B) atomicAdd(y + (size_t)b * R + row, yacc[t] * inv_xsc[b]);
      }
    }
#ifdef GSDLQ_TRACE
    if (trd) GSDLQ_TR_SET(0u, 26, tr_now());
#endif
  }
  // ---- release the tensor memory ----
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TCOLS);
  }
}

// The work buffer: per-token maxima ([0, 512)), per-token low-rank projections ([512, 8704)), from
// MM_XS_OFF the converted activations (one B tile per k-block), then the transposed fp32 activations.
constexpr size_t MM_XS_OFF = 16384;
inline size_t mm_xs_bytes(int nb, int cols) { return (size_t)(cols / MM_KB) * (size_t)(16 * nb * 128); }
inline size_t mm_work_bytes(int batch, int cols) {
  const int nb = (batch + 7) / 8;
  return MM_XS_OFF + mm_xs_bytes(nb, cols) + sizeof(float) * (size_t)cols * 8 * nb;
}

template <int NB>
static cudaError_t hexmm_launch_nb(int tiles, int nkb, cudaStream_t s, uint8_t* xs, const float* x, int B,
                                   const uint8_t* codes, const uint16_t* scales, const float* xy, int n_pts,
                                   const uint16_t* U, int k, const uint32_t* rp, const uint16_t* kc, const float* kd,
                                   float* y, int R, int C, const unsigned* amax, const float* tmp) {
  // up to MM_SMALL_NB token groups: the small-batch kernel (integer A, a scale per k-block slot)
  constexpr bool SMALL = NB <= MM_SMALL_NB;
  constexpr int smem = mm_smem<NB>();
  void (*kern)(const uint8_t*, int, const uint8_t*, const uint16_t*, const float*, int, float*, int, int, int,
               const unsigned*);
  if constexpr (SMALL)
    kern = hexmm_small_kernel<NB>;
  else
    kern = hexmm_kernel<NB>;
  static std::atomic<bool> configured[64];  // per device: the dynamic shared-memory opt-in is done
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!configured[dev].load(std::memory_order_acquire)) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  const float* xT = reinterpret_cast<const float*>(xs + mm_xs_bytes(NB, C));
  hexmm_xs_sparse<NB, SMALL><<<nkb + (R + 7) / 8, 256, 0, s>>>(x, B, C, amax, xs, nkb, xT, R, rp, kc, kd, U, k, tmp,
                                                               y);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // k-runs per row tile: the split that minimises (waves of resident CTAs) x (k-blocks per run + the
  // set-up and epilogue, about two blocks' worth)
  const int slots = mm_per_sm<NB>() * num_sms();
  int nsplit = 1;
  long long best = -1;
  for (int ns = 1; ns <= std::min(nkb, 64); ++ns) {
    const long long cost = (long long)((tiles * ns + slots - 1) / slots) * ((nkb + ns - 1) / ns + 2);
    if (best < 0 || cost < best) best = cost, nsplit = ns;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(tiles, nsplit);
  cfg.blockDim = dim3(MM_ALL);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, (const uint8_t*)xs, B, codes, scales, xy, n_pts, y, R, C, nsplit, amax);
}

int num_sms();
int record_cuda_error(cudaError_t e);

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_hex2d_matmul_work_size(int batch, int cols, size_t* bytes) {
  if (!bytes || batch < 1 || batch > MM_MAXB || cols <= 0 || cols % 64 != 0 || cols > 65535) return GSDLQ_ERR_INVALID;
  *bytes = mm_work_bytes(batch, cols);
  return GSDLQ_OK;
}

// The GEMM call.  tmp_ext (batch 1 only): the caller's low-rank projection S (Vt x) of the token, used
// instead of computing it from S and Vt (the drop-in matvec's contract, whose caller ran
// gsdlq_lowrank_proj).
static int hexmm_entry(const float* x, int batch, const uint8_t* codes, const uint16_t* scales,
                       const float* xy_table, const uint16_t* U, const float* S, const uint16_t* Vt,
                       const uint32_t* kink_row_ptr, const uint16_t* kink_cols, const float* kink_deltas, float* y,
                       void* work, size_t work_bytes, int rows, int cols, int k_dim, int n_pts, cudaStream_t s,
                       const float* tmp_ext) {
  if (!x || !codes || !scales || !xy_table || !kink_row_ptr || !y || !work) return GSDLQ_ERR_INVALID;
  if (batch < 1 || batch > MM_MAXB || rows <= 0 || cols <= 0 || cols % 64 != 0 || cols > 65535) return GSDLQ_ERR_INVALID;
  if (k_dim < 0 || k_dim > 16) return GSDLQ_ERR_INVALID;
  if (tmp_ext ? batch != 1 || (k_dim > 0 && !U) : k_dim > 0 && (!U || !S || !Vt)) return GSDLQ_ERR_INVALID;
  if (n_pts < 1 || n_pts > 256) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(codes) & 15u) return GSDLQ_ERR_INVALID;  // 16-byte code loads
  if ((reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(U)) & 1u) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(Vt) & 15u) return GSDLQ_ERR_INVALID;  // 16-byte loads of Vt rows
  if (reinterpret_cast<uintptr_t>(x) & 15u) return GSDLQ_ERR_INVALID;  // 16-byte activation loads
  if ((reinterpret_cast<uintptr_t>(y) & 3u) || (reinterpret_cast<uintptr_t>(work) & 1023u)) return GSDLQ_ERR_INVALID;
  if (work_bytes < mm_work_bytes(batch, cols)) return GSDLQ_ERR_INVALID;
  unsigned* amax = reinterpret_cast<unsigned*>(work);  // per-token max|x| (bits)
  float* tmp = reinterpret_cast<float*>(work) + MM_MAXB;
  uint8_t* xs = static_cast<uint8_t*>(work) + MM_XS_OFF;  // converted activations
  cudaError_t e = cudaMemsetAsync(work, 0, sizeof(float) * 17 * MM_MAXB, s);
  if (e != cudaSuccess) return record_cuda_error(e);
  if (tmp_ext && k_dim > 0) {  // token 0's projection slot: tmp[j], j < k_dim
    e = cudaMemcpyAsync(tmp, tmp_ext, sizeof(float) * k_dim, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  {
    const int nb = (batch + 7) / 8;
    float* xT = reinterpret_cast<float*>(static_cast<uint8_t*>(work) + MM_XS_OFF + mm_xs_bytes(nb, cols));
    // with tmp_ext the prep pass only converts x (k = 0: no projection of its own)
    hexmm_prep<<<dim3(nb, (cols + MM_PREP - 1) / MM_PREP), 256, 0, s>>>(
        x, batch, cols, tmp_ext ? nullptr : Vt, S, tmp_ext ? 0 : k_dim, amax, tmp, xT, 8 * nb, y, (size_t)batch * rows);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return record_cuda_error(e);
  const int tiles = (rows + MM_ROWS - 1) / MM_ROWS, nkb = cols / MM_KB;
  const float* kd = kink_deltas;
#define GSDLQ_MM_CASE(nb)                                                                                               \
  case nb:                                                                                                              \
    e = hexmm_launch_nb<nb>(tiles, nkb, s, xs, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr,     \
                            kink_cols, kd, y, rows, cols, amax, tmp);                                                   \
    break;
  switch ((batch + 7) / 8) {
    GSDLQ_MM_CASE(1) GSDLQ_MM_CASE(2) GSDLQ_MM_CASE(3) GSDLQ_MM_CASE(4) GSDLQ_MM_CASE(5) GSDLQ_MM_CASE(6)
    GSDLQ_MM_CASE(7) GSDLQ_MM_CASE(8) GSDLQ_MM_CASE(9) GSDLQ_MM_CASE(10) GSDLQ_MM_CASE(11) GSDLQ_MM_CASE(12)
    GSDLQ_MM_CASE(13) GSDLQ_MM_CASE(14) GSDLQ_MM_CASE(15) default: GSDLQ_MM_CASE(16)
  }
#undef GSDLQ_MM_CASE
  if (e != cudaSuccess) return record_cuda_error(e);
  return GSDLQ_OK;
}

extern "C" int gsdlq_hex2d_matmul(const float* x, int batch, const uint8_t* codes, const uint16_t* scales,
                                  const float* xy_table, const uint16_t* U, const float* S, const uint16_t* Vt,
                                  const uint32_t* kink_row_ptr, const uint16_t* kink_cols, const float* kink_deltas,
                                  float* y, void* work, size_t work_bytes, int rows, int cols, int k_dim, int n_pts,
                                  gsdlq_stream_t stream) {
  return hexmm_entry(x, batch, codes, scales, xy_table, U, S, Vt, kink_row_ptr, kink_cols, kink_deltas, y, work,
                     work_bytes, rows, cols, k_dim, n_pts, static_cast<cudaStream_t>(stream), nullptr);
}

namespace gsdlq {

// The drop-in matvec of a matrix the fused batch-1 kernel cannot plan (rows wider than its shared
// memory holds, or more strips than its per-CTA accumulator covers): this GEMM with one token and the
// caller's low-rank projection.  work: 1024-byte aligned, hexmm_wide_work_bytes(cols) bytes; x is first
// copied to its end, where the GEMM's 16-byte activation loads are aligned whatever the caller's x.
size_t hexmm_wide_work_bytes(int cols) { return mm_work_bytes(1, cols) + sizeof(float) * (size_t)cols; }

int hexmm_matvec_wide(const float* x, const uint8_t* codes, const uint16_t* scales, const float* xy_table,
                      const uint16_t* U, const float* tmp_k, const uint32_t* kink_row_ptr, const uint16_t* kink_cols,
                      const float* kink_deltas, float* y, void* work, int rows, int cols, int k_dim, int n_pts,
                      cudaStream_t s) {
  if (!x || !work || cols <= 0 || cols % 64 != 0 || cols > 65535 || (k_dim > 0 && !tmp_k)) return GSDLQ_ERR_INVALID;
  float* xa = reinterpret_cast<float*>(static_cast<uint8_t*>(work) + mm_work_bytes(1, cols));
  const cudaError_t e = cudaMemcpyAsync(xa, x, sizeof(float) * (size_t)cols, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return record_cuda_error(e);
  return hexmm_entry(xa, 1, codes, scales, xy_table, U, nullptr, nullptr, kink_row_ptr, kink_cols, kink_deltas, y,
                     work, mm_work_bytes(1, cols), rows, cols, k_dim, n_pts, s, tmp_k);
}

}  // namespace gsdlq

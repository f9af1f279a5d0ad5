// hexmm.cu -- the batched packed linear: B <= 128 tokens through one GSD-LQ matrix as a dequant-GEMM on
// the 5th-generation tensor cores (tcgen05, accumulators in tensor memory) -- the batch-B counterpart of
// gsd_cpu_lowrank_proj + gsd_cpu_hex2d_matvec (gsd_lq_cpu_engine.c:111-183) applied to each token, used
// for batched decode and for chunked prefill.
//
//   y[b][r] = sum_c W[r][c] x[b][c] + sum_{kinks of r} delta * x[b][col] + sum_j U[r][j] tmp[b][j],
//   W[r][2p + i] = xy[code(r, p)][i] * scale(r, p / 32),  tmp[b][j] = S[j] * (Vt[j] . x[b]).
//
// Layout of the work.  A CTA of 4 warps owns a tile of 128 weight rows and a contiguous run of 64-column
// k-blocks (split-K over CTAs, so that every SM streams weights).  Per k-block, through two shared-memory
// stages:
//   - thread t decodes the 32 code bytes of row t (one scale group) through a 256-entry float2 table into
//     fp32 weights, W = xy * scale as the reference's dequant defines them, splits them into fp16 hi + lo
//     parts (about 22 significant bits together) and writes them as two A operands in the K-major
//     128-byte-swizzle layout (a row's 64 columns are 128 bytes, 8 rows form a 1024-byte atom, 16-byte
//     chunk j of row r sits at chunk j ^ (r % 8), so the tensor core's reads spread over all banks);
//   - the block's activations of every token are written as the B operand in the same layout, token b as
//     two rows: 2b = fp16 hi, 2b + 1 = fp16 lo of x_b scaled by a power of two that puts max|x_b| in
//     [2^14, 2^15) (so both halves stay normal; about 22 significant bits together);
//   - one thread issues eight tcgen05.mma (W hi and W lo for each 16-column k-step; M = 128, N = 2 x tokens
//     padded to 8, fp16 in, fp32 accumulate in tensor memory) and commits them to the stage's mbarrier,
//     which releases the stage for the block two ahead; the next block's codes are loaded meanwhile.
// At the end each warp reads its 32 tensor-memory lanes (its rows) with tcgen05.ld, adds each token's hi
// and lo columns, unscales, and adds the partial sums into y (zeroed by the entry point) with fp32 atomics,
// so the summation order over the k-runs is not fixed.  The kink and low-rank terms are added once per
// (row, token) by the CTA whose run index equals the token index modulo the number of runs.
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "common.cuh"

namespace gsdlq {

constexpr int MM_ROWS = 128;      // weight rows per CTA (tensor-memory lanes)
constexpr int MM_KB = 64;         // columns per k-block: one scale group
constexpr int MM_THREADS = 256;   // two threads per weight row (its two 32-column halves of a block)
constexpr int MM_MAXB = GSDLQ_MATMUL_MAX_BATCH;  // tokens per call (N = 2 * 128 = 256, the largest MMA N)
constexpr int MM_AHALF = MM_ROWS * MM_KB * 2;  // bytes of one fp16 A tile (16 KB): the weights' hi or lo parts
constexpr int MM_ATILE = 2 * MM_AHALF;         // one stage's A tiles (hi, then lo)
constexpr int MM_HDR = 12288;                  // table, barriers, tensor-memory slot, token scales, projections

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
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
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
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);  // a in the low half
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int NB>
constexpr int mm_tcols() {  // tensor-memory columns of the accumulator: a power of two >= 32
  return 16 * NB <= 32 ? 32 : 16 * NB <= 64 ? 64 : 16 * NB <= 128 ? 128 : 256;
}
constexpr int MM_CSTAGES = 4;                  // k-blocks of codes in flight per CTA (cp.async ring)
constexpr int MM_CSTAGE = MM_ROWS * 32;        // code bytes of one k-block of a tile (4 KB)
template <int NB>
constexpr int mm_btile() {  // one k-block of the B operand: 16 NB rows (token hi / lo) x 128 bytes
  return 16 * NB * 128;
}
template <int NB>
constexpr int mm_smem() {
  // header + code ring + alignment slack + two A stages + two B stages; with 256 accumulator columns at
  // least 80 KB, so that no more than two CTAs share an SM's 512 tensor-memory columns (a third would
  // wait in tcgen05.alloc)
  constexpr int need = MM_HDR + MM_CSTAGES * MM_CSTAGE + 1024 + 2 * MM_ATILE + 2 * mm_btile<NB>();
  return (mm_tcols<NB>() == 256 && need < 80 * 1024) ? 80 * 1024 : need;
}
template <int NB>
constexpr bool mm_tmem_fits() {  // the CTAs that shared memory lets an SM hold fit its 512 tensor-memory columns
  return (227 * 1024 / mm_smem<NB>()) * mm_tcols<NB>() <= 512;
}
static_assert(mm_tmem_fits<1>() && mm_tmem_fits<2>() && mm_tmem_fits<3>() && mm_tmem_fits<4>() && mm_tmem_fits<5>() &&
                  mm_tmem_fits<6>() && mm_tmem_fits<7>() && mm_tmem_fits<8>() && mm_tmem_fits<9>() &&
                  mm_tmem_fits<12>() && mm_tmem_fits<16>(),
              "at most 512 tensor-memory columns of resident CTAs per SM");

// The B operand of every k-block, made once per call: token b's row of the block as fp16 hi (row 2b) and
// lo (row 2b + 1) of x_b scaled by its power of two, in the swizzled layout of a 64-column tile, one
// contiguous block of mm_btile<NB>() bytes per k-block (tokens past the batch are zero).
template <int NB>
__global__ void __launch_bounds__(256) hexmm_xconv(const float* __restrict__ x, int B, int C,
                                                   const unsigned* __restrict__ amax_bits, uint8_t* __restrict__ xs) {
  constexpr int BP = 8 * NB;
  const int kb = blockIdx.x;
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

// NB: groups of 8 tokens (tokens padded to 8 NB with zero activations); N = 16 NB accumulator columns.
// Thread t decodes half t / 128 of weight row t % 128 (32 columns of each 64-column block); warps 0-3
// read the accumulator lanes of rows 0-127 at the end.
template <int NB>
__global__ void __launch_bounds__(MM_THREADS) hexmm_kernel(const uint8_t* __restrict__ xs, const float* __restrict__ x,
                                                           int B, const uint8_t* __restrict__ codes,
                                                           const uint16_t* __restrict__ scales,
                                                           const float* __restrict__ xy, int n_pts,
                                                           const uint16_t* __restrict__ U, int k,
                                                           const uint32_t* __restrict__ row_ptr,
                                                           const uint16_t* __restrict__ kcols,
                                                           const float* __restrict__ kdel, float* __restrict__ y,
                                                           int R, int C, int nsplit, const unsigned* __restrict__ amax_bits,
                                                           const float* __restrict__ tmp) {
  constexpr int N = 16 * NB, BP = 8 * NB;
  constexpr uint32_t TCOLS = (uint32_t)mm_tcols<NB>();
  constexpr int BTILE = mm_btile<NB>();
  extern __shared__ __align__(1024) uint8_t sm[];
  float2* tab = reinterpret_cast<float2*>(sm);                    // [0, 2048)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 2080);       // tensor-memory address
  float* xsc = reinterpret_cast<float*>(sm + 2096);               // [MM_MAXB] token scales
  float* s_tmp = reinterpret_cast<float*>(sm + 2608);             // [BP][16] low-rank projections
  uint8_t* ring = sm + MM_HDR;                                    // code ring: [stage][row][32 bytes]
  const uint32_t sbase = smem_u32(sm);
  const uint32_t mbar = sbase + 2048, bbar = sbase + 2064;        // MMA-done and B-landed barriers, 2 each
  // the operand tiles start on a 1024-byte boundary of the shared window (the swizzle atoms' alignment)
  const uint32_t a_base = (sbase + MM_HDR + MM_CSTAGES * MM_CSTAGE + 1023u) & ~1023u;
  const uint32_t b_base = a_base + 2 * MM_ATILE;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int lr = tid & (MM_ROWS - 1), half = tid >> 7;  // weight row in the tile, column half of a block
  const int r0 = blockIdx.x * MM_ROWS, split = blockIdx.y;
  const int NP = C / 2, G = C / 64, nkb = C / MM_KB;
  const int kb0 = (int)((long long)nkb * split / nsplit), kb1 = (int)((long long)nkb * (split + 1) / nsplit);
  const int nk = kb1 - kb0;
  const int row = r0 + lr;
  const bool rok = row < R;
  const uint8_t* cp = codes + (size_t)(rok ? row : 0) * NP + half * 16;
  const uint16_t* scp = scales + (size_t)(rok ? row : 0) * G;
  // this thread's 16 code bytes of k-block kb0 + i into ring stage i % MM_CSTAGES (one group per block,
  // empty past the run, so that the group count stays uniform)
  auto fetch = [&](int i) {
    if (i < nk && rok) cp_async_16(ring + (i % MM_CSTAGES) * MM_CSTAGE + lr * 32 + half * 16, cp + (kb0 + i) * 32);
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < MM_CSTAGES - 1; ++i) fetch(i);

  for (int i = tid; i < 256; i += MM_THREADS) tab[i] = i < n_pts ? make_float2(xy[2 * i], xy[2 * i + 1]) : make_float2(0.f, 0.f);
  for (int i = tid; i < BP; i += MM_THREADS) xsc[i] = i < B ? hexmm_xscale(amax_bits[i]) : 0.f;
  for (int i = tid; i < BP * 16; i += MM_THREADS) s_tmp[i] = (i >> 4) < B ? tmp[i] : 0.f;
  if (tid == 0) {
    mbar_init(mbar, 1u);
    mbar_init(mbar + 8u, 1u);
    mbar_init(bbar, 1u);
    mbar_init(bbar + 8u, 1u);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);
#ifdef GSDLQ_TRACE
  // diagnostic builds: CTA blockIdx.x (< 160, run 0) stamps its set-up and its first six k-blocks
  const bool trc = blockIdx.y == 0 && tid == 0;
  if (trc) GSDLQ_TR_SET(0u, 0, tr_now());
#endif

  // The row's kinks (CSR, ascending columns) are added to their decoded weights in the A tiles, so the
  // tensor cores apply them with the lattice part.  e walks the row's list from this run's first column
  // (found in batches of eight independent loads); (kc, kd) is the kink at e and (kc2, kd2) the one after
  // it, loaded ahead so that the next block's test does not wait on a load.
  uint32_t e = rok ? row_ptr[row] : 0u;
  const uint32_t e_end = rok ? row_ptr[row + 1] : 0u;
  while (e < e_end) {
    int c8[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) c8[q] = e + q < e_end ? (int)kcols[e + q] : 0x7fffffff;
    int below = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) below += c8[q] < kb0 * MM_KB;
    e += below;
    if (below < 8) break;
  }
  int kc = e < e_end ? (int)kcols[e] : 0x7fffffff;
  float kd = e < e_end ? kdel[e] : 0.f;
  int kc2 = e + 1 < e_end ? (int)kcols[e + 1] : 0x7fffffff;
  float kd2 = e + 1 < e_end ? kdel[e + 1] : 0.f;

  uint16_t sc = (rok && nk > 0) ? scp[kb0] : (uint16_t)0;
  // instruction descriptor: D fp32, A and B fp16, both K-major, N, M = 128
  const uint32_t idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(MM_ROWS >> 4) << 24);
  bool bad = false;
  for (int i = 0; i < nk; ++i) {
    const int st = i & 1, kb = kb0 + i;
    // the MMAs of two blocks ago read this stage's A and B tiles: wait for their commit (bounded)
    if (i >= 2) mbar_wait_bounded(mbar + 8u * st, (uint32_t)(((i >> 1) - 1) & 1));
#ifdef GSDLQ_TRACE
    if (trc && i < 6) GSDLQ_TR_SET(0u, 1 + 4 * i, tr_now());
#endif
    if (tid == 0) {  // this block's B tile: one bulk copy from the converted activations
      mbar_arrive_expect_tx(bbar + 8u * st, (uint32_t)BTILE);
      bulk_g2s(b_base + st * BTILE, xs + (size_t)kb * BTILE, (uint32_t)BTILE, bbar + 8u * st);
    }
    fetch(i + MM_CSTAGES - 1);          // codes of the block MM_CSTAGES - 1 ahead
    cp_async_wait<MM_CSTAGES - 1>();    // this thread's codes of block i have landed
    // ---- A: 32 weights of row lr, chunks j = 4 half + jj (weights 8j .. 8j+7 = code bytes 4j .. 4j+3) ----
    const float s = h2f(sc);
    const uint4 cw = *reinterpret_cast<const uint4*>(ring + (i % MM_CSTAGES) * MM_CSTAGE + lr * 32 + half * 16);
    if (rok && i + 1 < nk) sc = scp[kb + 1];
    const uint32_t cv[4] = {cw.x, cw.y, cw.z, cw.w};
    uint8_t* atile = sm + (a_base - sbase) + st * MM_ATILE;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      uint32_t h[4], l[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int code = rok ? (int)((cv[jj] >> (8 * q)) & 0xffu) : 0;
        bad |= code >= n_pts;
        const float2 p = tab[code];
        const float w0 = p.x * s, w1 = p.y * s;  // a3 dequant: one fp32 multiply per weight
        const __half2 hh = __floats2half2_rn(w0, w1);
        h[q] = *reinterpret_cast<const uint32_t*>(&hh);
        l[q] = pack_h2(w0 - __low2float(hh), w1 - __high2float(hh));  // fp16 hi + lo: about 22 bits
      }
      *reinterpret_cast<uint4*>(atile + sw128(lr, 4 * half + jj)) = make_uint4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<uint4*>(atile + MM_AHALF + sw128(lr, 4 * half + jj)) = make_uint4(l[0], l[1], l[2], l[3]);
    }
    // the block's kinks in this thread's half: the weight's hi + lo halves plus the delta, split again (a
    // column repeated in the list gets every delta); kinks of the other half are the other thread's
    while (kc < (kb + 1) * MM_KB) {
      const int lc = kc - kb * MM_KB;  // 0 .. 63
      if ((lc >> 5) == half) {
        const int off = sw128(lr, lc >> 3) + 2 * (lc & 7);
        __half* ph = reinterpret_cast<__half*>(atile + off);
        __half* pl = reinterpret_cast<__half*>(atile + MM_AHALF + off);
        const float w = (__half2float(*ph) + __half2float(*pl)) + kd;
        const __half hw = __float2half_rn(w);
        *ph = hw;
        *pl = __float2half_rn(w - __half2float(hw));
      }
      ++e;
      kc = kc2;
      kd = kd2;
      kc2 = e + 1 < e_end ? (int)kcols[e + 1] : 0x7fffffff;
      kd2 = e + 1 < e_end ? kdel[e + 1] : 0.f;
    }
#ifdef GSDLQ_TRACE
    if (trc && i < 6) GSDLQ_TR_SET(0u, 2 + 4 * i, tr_now());
#endif
    fence_proxy_async_smem();  // the A tiles' generic stores, visible to the tensor core's reads
    mbar_wait_bounded(bbar + 8u * st, (uint32_t)((i >> 1) & 1));  // the B tile has landed
#ifdef GSDLQ_TRACE
    if (trc && i < 6) GSDLQ_TR_SET(0u, 3 + 4 * i, tr_now());
#endif
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < MM_KB / 16; ++kk) {
        const uint64_t bd = umma_desc(b_base + st * BTILE + kk * 32);
        umma_f16(tmem, umma_desc(a_base + st * MM_ATILE + kk * 32), bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_f16(tmem, umma_desc(a_base + st * MM_ATILE + MM_AHALF + kk * 32), bd, idesc, 1u);
      }
      umma_commit(mbar + 8u * st);  // arrives when every MMA issued so far has completed
#ifdef GSDLQ_TRACE
      if (trc && i < 6) GSDLQ_TR_SET(0u, 4 + 4 * i, tr_now());
#endif
    }
  }
  cp_async_wait<0>();
  if (bad) raise_flag(GSDLQ_FLAG_BAD_CODE);
  // a kink past the last column is never applied: the run that ends the row reports it
  if (kb1 == nkb && half == 0 && e < e_end) raise_flag(GSDLQ_FLAG_BAD_KINK);
#ifdef GSDLQ_TRACE
  if (trc) GSDLQ_TR_SET(0u, 25, tr_now());
#endif
  // ---- the run's partial sums: warps 0-3, lane = row; columns 2b, 2b + 1 = token b's hi and lo parts; the
  // low-rank term U[row] . tmp[b] is added once per (row, token), by the run whose index is b mod nsplit ----
  if (nk > 0 && warp < 4) {
    float u[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) u[j] = (rok && j < k) ? h2f(U[(size_t)row * k + j]) : 0.f;
    mbar_wait_bounded(mbar + 8u * ((nk - 1) & 1), (uint32_t)(((nk - 1) >> 1) & 1));
    tc_fence_after();
#pragma unroll 1
    for (int cb = 0; cb < N / 16; ++cb) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(cb * 16), v);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int b = cb * 8 + t;
        if (rok && b < B) {
          float val = (__uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1])) / xsc[b];
          if (b % nsplit == split) {
            float lrv = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) lrv = fmaf(u[j], s_tmp[b * 16 + j], lrv);
            val += lrv;
          }
          atomicAdd(y + (size_t)b * R + row, val);
        }
      }
    }
  }
#ifdef GSDLQ_TRACE
  if (trc) GSDLQ_TR_SET(0u, 26, tr_now());
  if (trc) {
    GSDLQ_TR_SET(0u, 27, tr_now());
    GSDLQ_TR_SET(0u, 28, (unsigned long long)nk);
  }
#endif
  // ---- release the tensor memory (every warp's loads are complete) ----
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TCOLS);
  }
}

// The work buffer: per-token maxima ([0, 512)), per-token low-rank projections ([512, 8704)), and from
// MM_XS_OFF the converted activations, one B tile per k-block.
constexpr size_t MM_XS_OFF = 16384;
inline size_t mm_work_bytes(int batch, int cols) {
  const int nb = (batch + 7) / 8;
  return MM_XS_OFF + (size_t)(cols / MM_KB) * (size_t)(16 * nb * 128);
}

template <int NB>
static cudaError_t hexmm_launch_nb(int tiles, int nkb, cudaStream_t s, uint8_t* xs, const float* x, int B,
                                   const uint8_t* codes, const uint16_t* scales, const float* xy, int n_pts,
                                   const uint16_t* U, int k, const uint32_t* rp, const uint16_t* kc, const float* kd,
                                   float* y, int R, int C, const unsigned* amax, const float* tmp) {
  constexpr int smem = mm_smem<NB>();
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(hexmm_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  hexmm_xconv<NB><<<nkb, 256, 0, s>>>(x, B, C, amax, xs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // k-runs per row tile: the CTAs that fit an SM at once (shared memory) on every SM, at least one
  // k-block each
  const int per_sm = std::max(1, std::min(8, (227 * 1024) / smem));
  const int nsplit = std::max(1, std::min(nkb, (per_sm * num_sms() + tiles - 1) / tiles));
  hexmm_kernel<NB><<<dim3(tiles, nsplit), MM_THREADS, smem, s>>>(xs, x, B, codes, scales, xy, n_pts, U, k, rp, kc, kd,
                                                                 y, R, C, nsplit, amax, tmp);
  return cudaGetLastError();
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

extern "C" int gsdlq_hex2d_matmul(const float* x, int batch, const uint8_t* codes, const uint16_t* scales,
                                  const float* xy_table, const uint16_t* U, const float* S, const uint16_t* Vt,
                                  const uint32_t* kink_row_ptr, const uint16_t* kink_cols, const float* kink_deltas,
                                  float* y, void* work, size_t work_bytes, int rows, int cols, int k_dim, int n_pts,
                                  gsdlq_stream_t stream) {
  if (!x || !codes || !scales || !xy_table || !kink_row_ptr || !y || !work) return GSDLQ_ERR_INVALID;
  if (batch < 1 || batch > MM_MAXB || rows <= 0 || cols <= 0 || cols % 64 != 0 || cols > 65535) return GSDLQ_ERR_INVALID;
  if (k_dim < 0 || k_dim > 16 || (k_dim > 0 && (!U || !S || !Vt))) return GSDLQ_ERR_INVALID;
  if (n_pts < 1 || n_pts > 256) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(codes) & 15u) return GSDLQ_ERR_INVALID;  // 16-byte code loads
  if ((reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(U) | reinterpret_cast<uintptr_t>(Vt)) & 1u)
    return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(x) & 15u) return GSDLQ_ERR_INVALID;  // 16-byte activation loads
  if ((reinterpret_cast<uintptr_t>(y) & 3u) || (reinterpret_cast<uintptr_t>(work) & 1023u)) return GSDLQ_ERR_INVALID;
  if (work_bytes < mm_work_bytes(batch, cols)) return GSDLQ_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* amax = reinterpret_cast<unsigned*>(work);  // per-token max|x| (bits)
  float* tmp = reinterpret_cast<float*>(work) + MM_MAXB;
  uint8_t* xs = static_cast<uint8_t*>(work) + MM_XS_OFF;  // converted activations
  cudaError_t e = cudaMemsetAsync(y, 0, sizeof(float) * (size_t)batch * rows, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(work, 0, sizeof(float) * 17 * MM_MAXB, s);
  if (e != cudaSuccess) return record_cuda_error(e);
  hexmm_prep<<<dim3(batch, (cols + MM_PREP - 1) / MM_PREP), 256, 0, s>>>(x, cols, Vt, S, k_dim, amax, tmp);
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

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
constexpr int MM_THREADS = 128;   // thread t decodes row t and reads lane t of the accumulator
constexpr int MM_MAXB = GSDLQ_MATMUL_MAX_BATCH;  // tokens per call (N = 2 * 128 = 256, the largest MMA N)
static_assert(GSDLQ_MATMUL_WORK_FLOATS >= 17 * MM_MAXB, "work: maxima and low-rank projections of every token");
constexpr int MM_AHALF = MM_ROWS * MM_KB * 2;  // bytes of one fp16 A tile (16 KB): the weights' hi or lo parts
constexpr int MM_ATILE = 2 * MM_AHALF;         // one stage's A tiles (hi, then lo)
constexpr int MM_HDR = 4096;                   // table, barriers, tensor-memory slot, token scales

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
template <int NB>
constexpr int mm_smem() {
  // header + two A stages + two B stages (16 NB rows of 128 bytes); with 256 accumulator columns at
  // least 80 KB, so that no more than two CTAs share an SM's 512 tensor-memory columns (a third
  // would wait in tcgen05.alloc)
  constexpr int need = MM_HDR + 1024 + 2 * MM_ATILE + 2 * 16 * NB * 128;  // (+1 KB: the tiles' alignment)
  return (mm_tcols<NB>() == 256 && need < 80 * 1024) ? 80 * 1024 : need;
}
static_assert(mm_smem<3>() * 9 > 227 * 1024 && mm_smem<5>() * 5 > 227 * 1024 && mm_smem<9>() * 3 > 227 * 1024,
              "at most 512 tensor-memory columns of resident CTAs per SM");

// NB: groups of 8 tokens (tokens padded to 8 NB with zero activations); N = 16 NB accumulator columns.
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
  constexpr int N = 16 * NB, BP = 8 * NB;
  constexpr uint32_t TCOLS = (uint32_t)mm_tcols<NB>();
  constexpr int BTILE = N * 128;
  extern __shared__ __align__(1024) uint8_t sm[];
  float2* tab = reinterpret_cast<float2*>(sm);                    // [0, 2048)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 2064);       // tensor-memory address
  float* xsc = reinterpret_cast<float*>(sm + 2080);               // [MM_MAXB] token scales
  const uint32_t sbase = smem_u32(sm);
  const uint32_t bar0 = sbase + 2048;                             // two mbarriers (8 bytes each)
  // the operand tiles start on a 1024-byte boundary of the shared window (the swizzle atoms' alignment)
  const uint32_t a_base = (sbase + MM_HDR + 1023u) & ~1023u, b_base = a_base + 2 * MM_ATILE;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int r0 = blockIdx.x * MM_ROWS, split = blockIdx.y;
  const int NP = C / 2, G = C / 64, nkb = C / MM_KB;
  const int kb0 = (int)((long long)nkb * split / nsplit), kb1 = (int)((long long)nkb * (split + 1) / nsplit);
  const int nk = kb1 - kb0;

  for (int i = tid; i < 256; i += MM_THREADS) tab[i] = i < n_pts ? make_float2(xy[2 * i], xy[2 * i + 1]) : make_float2(0.f, 0.f);
  for (int i = tid; i < BP; i += MM_THREADS) xsc[i] = i < B ? hexmm_xscale(amax_bits[i]) : 0.f;
  if (tid == 0) {
    mbar_init(bar0, 1u);
    mbar_init(bar0 + 8u, 1u);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);

  const int row = r0 + tid;
  const bool rok = row < R;
  const uint8_t* cp = codes + (size_t)(rok ? row : 0) * NP;
  const uint16_t* scp = scales + (size_t)(rok ? row : 0) * G;
  uint4 c0 = make_uint4(0u, 0u, 0u, 0u), c1 = make_uint4(0u, 0u, 0u, 0u);
  uint16_t sc = 0;
  if (rok && nk > 0) {
    c0 = *reinterpret_cast<const uint4*>(cp + kb0 * 32);
    c1 = *reinterpret_cast<const uint4*>(cp + kb0 * 32 + 16);
    sc = scp[kb0];
  }
  // instruction descriptor: D fp32, A and B fp16, both K-major, N, M = 128
  const uint32_t idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(MM_ROWS >> 4) << 24);
  bool bad = false;
  for (int kb = kb0; kb < kb1; ++kb) {
    const int i = kb - kb0, st = i & 1;
    // the MMAs of two blocks ago read this stage: wait for their commit (bounded)
    if (i >= 2) mbar_wait_bounded(bar0 + 8u * st, (uint32_t)(((i >> 1) - 1) & 1));
    // ---- A: row tid's 64 weights, chunk j = weights 8j .. 8j+7 = code bytes 4j .. 4j+3 ----
    const float s = h2f(sc);
    const uint32_t cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    uint8_t* atile = sm + (a_base - sbase) + st * MM_ATILE;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t h[4], l[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int code = (int)((cv[j] >> (8 * q)) & 0xffu);
        bad |= rok && code >= n_pts;
        const float2 p = tab[code];
        const float w0 = p.x * s, w1 = p.y * s;  // a3 dequant: one fp32 multiply per weight
        const __half2 hh = __floats2half2_rn(w0, w1);
        h[q] = *reinterpret_cast<const uint32_t*>(&hh);
        l[q] = pack_h2(w0 - __low2float(hh), w1 - __high2float(hh));  // fp16 hi + lo: about 22 bits
      }
      *reinterpret_cast<uint4*>(atile + sw128(tid, j)) = make_uint4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<uint4*>(atile + MM_AHALF + sw128(tid, j)) = make_uint4(l[0], l[1], l[2], l[3]);
    }
    // the next block's codes into registers while this one is staged and multiplied
    if (rok && kb + 1 < kb1) {
      c0 = *reinterpret_cast<const uint4*>(cp + (kb + 1) * 32);
      c1 = *reinterpret_cast<const uint4*>(cp + (kb + 1) * 32 + 16);
      sc = scp[kb + 1];
    }
    // ---- B: token b, chunk j -> rows 2b (hi) and 2b + 1 (lo) ----
    uint8_t* bt = sm + (b_base - sbase) + st * BTILE;
    for (int e = tid; e < BP * 8; e += MM_THREADS) {
      const int b = e >> 3, j = e & 7;
      float v[8];
      if (b < B) {
        const float4* xp = reinterpret_cast<const float4*>(x + (size_t)b * C + kb * MM_KB + 8 * j);
        const float4 u0 = xp[0], u1 = xp[1];
        const float f = xsc[b];
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
      const int rh = 2 * b, rl = 2 * b + 1;
      *reinterpret_cast<uint4*>(bt + sw128(rh, j)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(bt + sw128(rl, j)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    fence_proxy_async_smem();  // the tiles' generic stores, visible to the tensor core's reads
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < MM_KB / 16; ++kk) {
        const uint64_t bd = umma_desc(b_base + st * BTILE + kk * 32);
        umma_f16(tmem, umma_desc(a_base + st * MM_ATILE + kk * 32), bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_f16(tmem, umma_desc(a_base + st * MM_ATILE + MM_AHALF + kk * 32), bd, idesc, 1u);
      }
      umma_commit(bar0 + 8u * st);  // arrives when every MMA issued so far has completed
    }
  }
  if (bad) raise_flag(GSDLQ_FLAG_BAD_CODE);
  // ---- the run's partial sums: lane tid = row tid; columns 2b, 2b + 1 = token b's hi and lo parts ----
  if (nk > 0) {
    mbar_wait_bounded(bar0 + 8u * ((nk - 1) & 1), (uint32_t)(((nk - 1) >> 1) & 1));
    tc_fence_after();
#pragma unroll 1
    for (int cb = 0; cb < N / 16; ++cb) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(cb * 16), v);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int b = cb * 8 + t;
        if (rok && b < B)
          atomicAdd(y + (size_t)b * R + row, (__uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1])) / xsc[b]);
      }
    }
  }
  // ---- kinks and the low-rank term, once per (row, token): tokens b = split (mod nsplit) ----
  bool badk = false;
  if (rok) {
    for (int b = split; b < B; b += nsplit) {
      float v = 0.f;
      for (int j = 0; j < k; ++j) v = fmaf(h2f(U[(size_t)row * k + j]), tmp[(size_t)b * 16 + j], v);
      const float* xb = x + (size_t)b * C;
      for (uint32_t e = row_ptr[row]; e < row_ptr[row + 1]; ++e) {
        const int col = kcols[e];
        if (col < C) v = fmaf(kdel[e], xb[col], v);
        else badk = true;
      }
      atomicAdd(y + (size_t)b * R + row, v);
    }
  }
  if (badk) raise_flag(GSDLQ_FLAG_BAD_KINK);
  // ---- release the tensor memory (every warp's loads are complete) ----
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TCOLS);
  }
}

template <int NB>
static cudaError_t hexmm_launch_nb(int tiles, int nkb, cudaStream_t s, const float* x, int B, const uint8_t* codes,
                                   const uint16_t* scales, const float* xy, int n_pts, const uint16_t* U, int k,
                                   const uint32_t* rp, const uint16_t* kc, const float* kd, float* y, int R, int C,
                                   const unsigned* amax, const float* tmp) {
  constexpr int smem = mm_smem<NB>();
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(hexmm_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  // k-runs per row tile: the CTAs that fit an SM at once (shared memory) on every SM, at least one
  // k-block each
  const int per_sm = std::max(1, std::min(8, (227 * 1024) / smem));
  const int nsplit = std::max(1, std::min(nkb, (per_sm * num_sms() + tiles - 1) / tiles));
  hexmm_kernel<NB><<<dim3(tiles, nsplit), MM_THREADS, smem, s>>>(x, B, codes, scales, xy, n_pts, U, k, rp, kc, kd, y, R,
                                                                 C, nsplit, amax, tmp);
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
  if (reinterpret_cast<uintptr_t>(x) & 15u) return GSDLQ_ERR_INVALID;  // 16-byte activation loads
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(work)) & 3u) return GSDLQ_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* amax = reinterpret_cast<unsigned*>(work);  // per-token max|x| (bits)
  float* tmp = work + MM_MAXB;
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
    e = hexmm_launch_nb<nb>(tiles, nkb, s, x, batch, codes, scales, xy_table, n_pts, U, k_dim, kink_row_ptr, kink_cols, \
                            kd, y, rows, cols, amax, tmp);                                                              \
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

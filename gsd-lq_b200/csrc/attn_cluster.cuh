// attn_cluster.cuh -- the stand-alone split-KV GQA decode attention on sm_100a
// (gsd_lq_cpu_engine.c:265-330): tensor-core score and P.V tiles, and one thread-block cluster
// per kv head whose CTAs combine their splits through distributed shared memory.
//
// Grid (AC_CL, n_kv_heads), cluster (AC_CL, 1, 1): CTA r of kv head h takes the r-th of AC_CL
// equal runs of whole 64-token tiles of positions [0, pos].  Its tiles' K and V rows are copied
// into shared memory when the CTA starts (they were written by earlier steps), the row at pos and
// q after the programmatic-dependent-launch wait (the QKV kernel writes them).
//
// Arithmetic per tile, all in fp32 accuracy:
//   scores S[t][h] = K[t] . q_h: mma.sync m16n8k16 with A = K rows (fp16, exact) and B = q split
//     into fp16 hi + lo (after scaling by a power of two that puts max|q| in [2^14, 2^15), so
//     both parts stay normal); S = (A.B_hi + A.B_lo) * sm_scale / scale;
//   softmax per head (one warp per head), P = exp(S - m) scaled by 2^11 and split into fp16 hi
//     (A rows 0..7) + lo (A rows 8..15): one pass over all of the CTA's tokens when its tiles fit
//     the AC_NBUF buffers (the common case: 8 warps take the score tiles, then one softmax and one
//     P.V sweep), else tile by tile with an online softmax;
//   O[h][d] += P . V: mma.sync with A = P rows, B = V rows read transposed by ldmatrix; rows g
//     (hi) and g + 8 (lo) of the accumulator are the same head, so their sum is the output.
// Combine: each CTA leaves (m_h, l_h, O_h) in its shared memory; after a cluster barrier CTA r
// reads the AC_CL copies of its 1/AC_CL slice of the outputs through distributed shared memory,
// rescales them by exp(m_c - max m), writes the slice and, when asked, forwards the O linear's
// low-rank projection of it.  A second cluster barrier keeps every CTA's shared memory alive
// until the others have read it.  Every thread of every CTA reaches both barriers: there is no
// early return anywhere in the kernel.
#pragma once
#include "attn_dev.cuh"

namespace gsdlq {

constexpr int AC_CL = 8;             // CTAs per kv head (one cluster)
constexpr int AC_THREADS = 256;
constexpr int AC_NBUF = 4;           // K/V tile buffers in shared memory
constexpr int AC_MAXK = 48;          // largest forwarded low-rank dimension
constexpr float AC_PSCALE = 2048.f;  // P is scaled by 2^11 before its fp16 split

template <int HD, int GQ>
struct AcLayout {
  static constexpr int ROWB = HD * 2 + 16;          // K/V row bytes, padded (conflict-free fragments)
  static constexpr int TILEB = 2 * AT_TILE * ROWB;  // K rows, then V rows
  static constexpr int QROW = HD + 8;               // halves per q row (padded)
  static constexpr int SPW = AC_NBUF * AT_TILE;     // score columns: every buffered token
  static constexpr int PROW = SPW + 8;              // halves per P row (padded)
  static constexpr int OPC = GQ * HD / AC_CL;       // outputs each CTA combines
  static constexpr int KV = 0;
  static constexpr int QS = KV + AC_NBUF * TILEB;   // fp16 [16][QROW]: q hi (rows 0..7), lo (8..15)
  static constexpr int PS = QS + 16 * QROW * 2;     // fp16 [16][PROW]: P hi (rows 0..7), lo (8..15)
  static constexpr int SP = PS + 16 * PROW * 2;     // fp32 [GQ][SPW]: scaled scores
  static constexpr int ACC = SP + GQ * SPW * 4;     // fp32 [GQ * HD]: this CTA's output x 2^11
  static constexpr int ST = ACC + GQ * HD * 4;      // fp32: m[8], l[8], f[8], reduction[8]
  static constexpr int VT = ST + 32 * 4;            // fp16 [AC_MAXK][OPC]: forwarded Vt slice
  static constexpr int FR = VT + AC_MAXK * OPC * 2; // fp32 [8 warps][16]: forward partial sums
  static constexpr int BYTES = FR + 8 * 16 * 4;
  static_assert(QS % 16 == 0 && PS % 16 == 0 && SP % 16 == 0 && ACC % 16 == 0 && VT % 16 == 0 && FR % 16 == 0,
                "shared-memory regions must stay 16-byte aligned");
};

// D += A(16x16 fp16, row) * B(16x8 fp16, col), fp32 accumulate
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two 8x8 fp16 matrices, transposed: lanes 0-7 address the rows of the first, 8-15 of the second
__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t& b0, uint32_t& b1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(b0), "=r"(b1)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// the address of the same shared-memory variable in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Sums 16 values over the 32 lanes of a warp in 16 shuffles (instead of 16 x 5): after the
// exchanges lane l holds the total of value (l >> 1) & 15.
__device__ __forceinline__ float warp_sum16(float (&v)[16], int lane) {
#pragma unroll
  for (int w = 8, bit = 16; w >= 1; w >>= 1, bit >>= 1) {
    const bool up = (lane & bit) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = up ? v[i] : v[i + w];
      const float keep = up ? v[i + w] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

template <int HD, int GQ>
__global__ void __launch_bounds__(AC_THREADS, 1) attn_cluster_kernel(const __grid_constant__ gsdlq_attn_job_t J) {
  using Lo = AcLayout<HD, GQ>;
  constexpr int ROWB = Lo::ROWB, CH = HD / 8, KS = HD / 16, QROW = Lo::QROW, PROW = Lo::PROW, OPC = Lo::OPC;
  constexpr int SPW = Lo::SPW;
  constexpr int NTALL = HD / 8;              // 8-dimension column tiles of the output
  constexpr int NTW = (NTALL + 7) / 8;       // column tiles per warp in P.V
  constexpr int NQ = (GQ * HD + AC_THREADS - 1) / AC_THREADS;
  extern __shared__ __align__(16) uint8_t sm[];
  uint16_t* qs = reinterpret_cast<uint16_t*>(sm + Lo::QS);
  uint16_t* ps = reinterpret_cast<uint16_t*>(sm + Lo::PS);
  float* sp = reinterpret_cast<float*>(sm + Lo::SP);
  float* accs = reinterpret_cast<float*>(sm + Lo::ACC);
  float* s_m = reinterpret_cast<float*>(sm + Lo::ST);
  float* s_l = s_m + 8;
  float* s_f = s_m + 16;
  float* red = s_m + 24;
  uint16_t* vts = reinterpret_cast<uint16_t*>(sm + Lo::VT);
  float* fr = reinterpret_cast<float*>(sm + Lo::FR);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q4 = lane & 3;
  const int rank = blockIdx.x;  // == the CTA's rank in its cluster (cluster dims (AC_CL, 1, 1))
  const int kvh = blockIdx.y;
  pdl_trigger_ops();  // the next launch may be scheduled at once (its wait covers this grid)

  const int pos = J.pos_dev ? *J.pos_dev : J.pos_val;
  const bool pos_ok = pos >= 0 && pos < J.max_seq;
  const int len = pos_ok ? pos + 1 : 0;
  const int tpc = AT_TILE * ((len + AC_CL * AT_TILE - 1) / (AC_CL * AT_TILE));  // tokens per CTA
  const int t0 = min(len, rank * tpc), t1 = min(len, t0 + tpc);
  const int ntiles = (t1 - t0 + AT_TILE - 1) / AT_TILE;
  const size_t tok_stride = (size_t)J.n_kv_heads * HD;
  auto row_off = [&](int t) -> size_t {
    const size_t slot = J.block_table ? (size_t)J.block_table[t / J.page_size] * J.page_size + (t % J.page_size)
                                      : (size_t)J.layer * J.max_seq + t;
    return slot * tok_stride + (size_t)kvh * HD;
  };
  auto tile_k = [&](int i) -> uint8_t* { return sm + Lo::KV + (i % AC_NBUF) * Lo::TILEB; };
  // copies of tile i's rows selected by `which` (0: < pos, 1: == pos, 2: all); the V rows past a
  // partial tile's end are zeroed (P is zero there, and 0 * NaN would not be)
  auto issue = [&](int i, int which) {
    const int tb = t0 + i * AT_TILE, nt = min(AT_TILE, t1 - tb);
    uint8_t* kb = tile_k(i);
    uint8_t* vb = kb + AT_TILE * ROWB;
    for (int e = tid; e < nt * CH; e += AC_THREADS) {
      const int j = e / CH, c = e - j * CH, t = tb + j;
      if (which == 2 || (which == 0 ? t < pos : t == pos)) {
        const size_t off = row_off(t) + c * 8;
        cp_async_16(kb + j * ROWB + c * 16, J.k_cache + off);
        cp_async_16(vb + j * ROWB + c * 16, J.v_cache + off);
      }
    }
    if (which != 1)
      for (int e = tid; e < (AT_TILE - nt) * (ROWB / 16); e += AC_THREADS)
        reinterpret_cast<uint4*>(vb + nt * ROWB)[e] = make_uint4(0u, 0u, 0u, 0u);
    cp_async_commit();
  };

  // ---- before the wait: operand padding, softmax state, the earlier rows, the Vt slice ----------
  for (int e = tid; e < (Lo::SP - Lo::QS) / 16; e += AC_THREADS)
    reinterpret_cast<uint4*>(sm + Lo::QS)[e] = make_uint4(0u, 0u, 0u, 0u);  // q and P rows of absent heads
  if (tid < 8) {
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.f;
    s_f[tid] = 0.f;
  }
  for (int i = 0; i < min(ntiles, AC_NBUF); ++i) issue(i, 0);
  // the later launches' weights go into L2 while attention runs (it reads little from HBM)
  if (warp == AC_THREADS / 32 - 1) issue_prefetch(J.prefetch, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y, lane);
  const int fk = J.fwd_acc != nullptr ? J.fwd_k : 0;
  const int col0 = kvh * GQ * HD + rank * OPC;  // this CTA's first output column of the O linear
  {
    const size_t n_in = (size_t)J.n_heads * HD;
    for (int e = tid; e < fk * (OPC / 2); e += AC_THREADS) {
      const int j = e / (OPC / 2), c = e - j * (OPC / 2);
      cp_async_4(vts + j * OPC + 2 * c, J.fwd_vt + (size_t)j * n_in + col0 + 2 * c);
    }
    cp_async_commit();
  }

  pdl_wait_ops();
  if (!pos_ok && tid == 0 && kvh == 0 && rank == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
  if (pos >= t0 && pos < t1 && (pos - t0) / AT_TILE < AC_NBUF) issue((pos - t0) / AT_TILE, 1);
  // q of this head group, scaled by a power of two and split into fp16 hi + lo
  float qv[NQ];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    const int i = tid + k * AC_THREADS;
    qv[k] = i < GQ * HD ? __ldcg(J.q + (size_t)kvh * GQ * HD + i) : 0.f;
    amax = fmaxf(amax, fabsf(qv[k]));
  }
  amax = warp_max(amax);
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  int qe = 0;
  frexpf(amax, &qe);                                   // amax < 2^qe
  qe = max(qe, -111);
  const float qscale = (amax > 0.f && amax <= 3.0e38f) ? ldexpf(1.f, 15 - qe) : 1.f;
  const float sscale = J.sm_scale / qscale;
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    const int i = tid + k * AC_THREADS;
    if (i < GQ * HD) {
      const int h = i / HD, d = i - h * HD;
      const float x = qv[k] * qscale;
      const uint16_t hi = f2h(x);
      qs[h * QROW + d] = hi;
      qs[(8 + h) * QROW + d] = f2h(x - h2f(hi));
    }
  }

  // ---- tiles ---------------------------------------------------------------------------------
  float acc[NTW][4];
#pragma unroll
  for (int n = 0; n < NTW; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  // scores of the 16 tokens from row rb of tile buffer kb against both q splits, into score
  // columns c0 .. c0+15; lane (g, q4) holds heads 2q4, 2q4+1 of tokens c0+g (c[0], c[1]) and
  // c0+g+8 (c[2], c[3])
  auto scores16 = [&](const uint8_t* kb, int rb, int c0) {
    float ch[4] = {0.f, 0.f, 0.f, 0.f}, cl[4] = {0.f, 0.f, 0.f, 0.f};
    const uint8_t* r0 = kb + (rb + g) * ROWB + 4 * q4;
    const uint8_t* r1 = r0 + 8 * ROWB;
    const uint16_t* qh = qs + g * QROW + 2 * q4;
    const uint16_t* ql = qh + 8 * QROW;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t a[4];
      a[0] = *reinterpret_cast<const uint32_t*>(r0 + kk * 32);
      a[1] = *reinterpret_cast<const uint32_t*>(r1 + kk * 32);
      a[2] = *reinterpret_cast<const uint32_t*>(r0 + kk * 32 + 16);
      a[3] = *reinterpret_cast<const uint32_t*>(r1 + kk * 32 + 16);
      mma_f16_16816(ch, a, *reinterpret_cast<const uint32_t*>(qh + kk * 16),
                    *reinterpret_cast<const uint32_t*>(qh + kk * 16 + 8));
      mma_f16_16816(cl, a, *reinterpret_cast<const uint32_t*>(ql + kk * 16),
                    *reinterpret_cast<const uint32_t*>(ql + kk * 16 + 8));
    }
    const int h0 = 2 * q4, ta = c0 + g;
    if (h0 < GQ) {
      sp[h0 * SPW + ta] = (ch[0] + cl[0]) * sscale;
      sp[h0 * SPW + ta + 8] = (ch[2] + cl[2]) * sscale;
    }
    if (h0 + 1 < GQ) {
      sp[(h0 + 1) * SPW + ta] = (ch[1] + cl[1]) * sscale;
      sp[(h0 + 1) * SPW + ta + 8] = (ch[3] + cl[3]) * sscale;
    }
  };
  // P.V over the first nk 16-token k-steps of the P columns; vrows(kk) is the first V row of
  // k-step kk.  Warp w takes output column tiles w*NTW .. w*NTW+NTW-1; accumulator rows g (P hi)
  // and g + 8 (P lo) both belong to head g.
  auto pv = [&](int nk, auto vrows) {
    if (warp * NTW < NTALL) {
      const uint16_t* p0 = ps + g * PROW + 2 * q4;
      const uint16_t* p1 = p0 + 8 * PROW;
#pragma unroll 4
      for (int kk = 0; kk < nk; ++kk) {
        uint32_t a[4];
        a[0] = *reinterpret_cast<const uint32_t*>(p0 + kk * 16);
        a[1] = *reinterpret_cast<const uint32_t*>(p1 + kk * 16);
        a[2] = *reinterpret_cast<const uint32_t*>(p0 + kk * 16 + 8);
        a[3] = *reinterpret_cast<const uint32_t*>(p1 + kk * 16 + 8);
        const uint8_t* vr = vrows(kk) + (lane & 15) * ROWB;
#pragma unroll
        for (int n = 0; n < NTW; ++n) {
          uint32_t b0, b1;
          ldsm_x2_trans(smem_u32(vr + (warp * NTW + n) * 16), b0, b1);
          mma_f16_16816(acc[n], a, b0, b1);
        }
      }
    }
  };
  if (ntiles > 0 && ntiles <= AC_NBUF) {
    // every tile is buffered: scores of all of them, one softmax per head, one P.V sweep
    const int ntot = t1 - t0;
    cp_async_wait_all();
    __syncthreads();
    for (int mt = warp; mt < 4 * ntiles; mt += 8) scores16(tile_k(mt >> 2), (mt & 3) * 16, mt * 16);
    __syncthreads();
    if (warp < GQ) {  // warp h: head h, token lane + 32 j
      const int h = warp;
      float v[SPW / 32];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < SPW / 32; ++j) {
        const int t = lane + 32 * j;
        v[j] = t < ntot ? sp[h * SPW + t] : -INFINITY;
        mx = fmaxf(mx, v[j]);
      }
      const float m = warp_max(mx);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < SPW / 32; ++j) {
        const int t = lane + 32 * j;
        const float e = t < ntot ? expf(v[j] - m) : 0.f;
        sum += e;
        const float x = e * AC_PSCALE;
        const uint16_t hi = f2h(x);
        ps[h * PROW + t] = hi;
        ps[(8 + h) * PROW + t] = f2h(x - h2f(hi));
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        s_m[h] = m;
        s_l[h] = sum;
      }
    }
    __syncthreads();
    pv(4 * ntiles, [&](int kk) { return tile_k(kk >> 2) + AT_TILE * ROWB + (kk & 3) * 16 * ROWB; });
  } else {
    // more tiles than buffers: tile by tile with an online softmax, refilling each buffer after use
    for (int i = 0; i < ntiles; ++i) {
      const int nt = min(AT_TILE, t1 - (t0 + i * AT_TILE));
      const uint8_t* kb = tile_k(i);
      const uint8_t* vb = kb + AT_TILE * ROWB;
      cp_async_wait_all();
      __syncthreads();
      if (warp < 4) scores16(kb, 16 * warp, 16 * warp);
      __syncthreads();
      // online softmax: warp h takes head h
      if (warp < GQ) {
        const int h = warp;
        const float a = lane < nt ? sp[h * SPW + lane] : -INFINITY;
        const float b = lane + 32 < nt ? sp[h * SPW + lane + 32] : -INFINITY;
        const float m_old = s_m[h];
        const float m = fmaxf(m_old, warp_max(fmaxf(a, b)));
        const float ea = lane < nt ? expf(a - m) : 0.f;
        const float eb = lane + 32 < nt ? expf(b - m) : 0.f;
        const float xa = ea * AC_PSCALE, xb = eb * AC_PSCALE;
        const uint16_t ha = f2h(xa), hb = f2h(xb);
        ps[h * PROW + lane] = ha;
        ps[h * PROW + lane + 32] = hb;
        ps[(8 + h) * PROW + lane] = f2h(xa - h2f(ha));
        ps[(8 + h) * PROW + lane + 32] = f2h(xb - h2f(hb));
        const float sum = warp_sum(ea + eb);
        if (lane == 0) {
          const float f = (m_old == -INFINITY) ? 0.f : expf(m_old - m);
          s_f[h] = f;
          s_m[h] = m;
          s_l[h] = s_l[h] * f + sum;
        }
      }
      __syncthreads();
      const float f = g < GQ ? s_f[g] : 0.f;  // rescale the running output by this tile's factor
#pragma unroll
      for (int n = 0; n < NTW; ++n) {
        acc[n][0] *= f;
        acc[n][1] *= f;
        acc[n][2] *= f;
        acc[n][3] *= f;
      }
      pv(AT_TILE / 16, [&](int kk) { return vb + kk * 16 * ROWB; });
      if (i + AC_NBUF < ntiles) {
        __syncthreads();  // every read of this buffer is done before it is refilled
        issue(i + AC_NBUF, 2);
      }
    }
  }
  // this CTA's output (x 2^11) for the combine; m = -inf, l = 0, O = 0 without tokens
  if (warp * NTW < NTALL && g < GQ) {
#pragma unroll
    for (int n = 0; n < NTW; ++n) {
      const int d = (warp * NTW + n) * 8 + 2 * q4;
      accs[g * HD + d] = acc[n][0] + acc[n][2];
      accs[g * HD + d + 1] = acc[n][1] + acc[n][3];
    }
  }
  cp_async_wait_all();  // (the Vt slice)
  cluster_sync_all();

  // ---- combine this CTA's slice of the kv head's outputs across the cluster -------------------
  float outv = 0.f;
  if (tid < OPC) {
    const int o = rank * OPC + tid, h = o / HD;
    const uint32_t a_acc = smem_u32(accs + o), a_m = smem_u32(s_m + h), a_l = smem_u32(s_l + h);
    float mc[AC_CL], lc[AC_CL], ac[AC_CL];
#pragma unroll
    for (int c = 0; c < AC_CL; ++c) {
      mc[c] = ld_cluster_f32(mapa_shared(a_m, c));
      lc[c] = ld_cluster_f32(mapa_shared(a_l, c));
      ac[c] = ld_cluster_f32(mapa_shared(a_acc, c));
    }
    float M = mc[0];
#pragma unroll
    for (int c = 1; c < AC_CL; ++c) M = fmaxf(M, mc[c]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int c = 0; c < AC_CL; ++c) {
      const float f = (mc[c] == -INFINITY) ? 0.f : expf(mc[c] - M);
      L = fmaf(lc[c], f, L);
      A = fmaf(ac[c], f, A);
    }
    outv = L > 0.f ? A / (L * AC_PSCALE) : 0.f;
    J.out[(size_t)kvh * GQ * HD + o] = outv;
  }
  // low-rank forwarding into the O linear: sum_o Vt[j][col0 + o] * out[o] over this slice
  for (int j0 = 0; j0 < fk; j0 += 16) {
    float v[16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj)
      v[jj] = (tid < OPC && j0 + jj < fk) ? h2f(vts[(j0 + jj) * OPC + tid]) * outv : 0.f;
    const float s = warp_sum16(v, lane);
    if ((lane & 1) == 0) fr[warp * 16 + ((lane >> 1) & 15)] = s;
    __syncthreads();
    if (tid < 16 && j0 + tid < fk) {
      float a = 0.f;
      for (int w = 0; w < (OPC + 31) / 32; ++w) a += fr[w * 16 + tid];
      if (!(fabsf(a) < 4194304.f)) {
        raise_flag(GSDLQ_FLAG_RANGE);
        a = (a != a) ? 0.f : copysignf(4194304.f, a);
      }
      atomicAdd(J.fwd_acc + j0 + tid, (unsigned long long)__float2ll_rn(a * 4294967296.f));
    }
    __syncthreads();
  }
  cluster_sync_all();  // the other CTAs may still be reading this CTA's shared memory
}

}  // namespace gsdlq

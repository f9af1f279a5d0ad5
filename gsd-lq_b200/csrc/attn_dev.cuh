// attn_dev.cuh -- device code of the split-KV GQA decode attention on sm_100a (gsd_lq_cpu_engine.c:265-330).
#pragma once
#include <algorithm>

#include "common.cuh"

namespace gsdlq {

// split-KV decode attention (flash-decoding).  CTA (kv head, split) processes its token range
// in tiles of AT_TILE rows: the K and V rows are staged in shared memory (row stride padded by
// 16 bytes so that 16-byte reads are conflict-free), four threads compute one token's scores
// for all GQ query heads of the group, a warp per head keeps the running softmax of the
// split, and each thread accumulates P.V for one dimension pair of one (or two) heads.  The
// split writes (max, sum, acc[hd]) per head; the last CTA of a kv head combines the splits
// (one batch of loads per output), or the only split writes the output itself.  Rows of
// positions < pos come from earlier steps, so the first tile's rows are loaded before the
// programmatic-dependent-launch wait; q and the row at pos (written by the QKV kernel) after.
// The same body serves the stand-alone kernel (one group = one CTA) and the persistent decode
// kernel, where each half of a CTA is a group with its own named barrier and the producer of q is
// a completion counter instead of the previous launch.
constexpr int AT_THREADS = 256;
constexpr int AT_TILE = 64;       // tokens per tile
constexpr int AT_MAX_GQ = 8;
constexpr int AT_MAX_SPLITS = 32;

// tokens per split: a multiple of the tile with at most AT_MAX_SPLITS splits
inline int attn_tokens_per_split(int max_seq) {
  const int span = AT_TILE * AT_MAX_SPLITS;
  return AT_TILE * std::max(1, (max_seq + span - 1) / span);
}

__device__ __forceinline__ void pdl_wait_ops() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_ops() { asm volatile("griddepcontrol.launch_dependents;"); }

template <int HD, int GQ>
struct __align__(16) AttnSmem {
  uint8_t skv[2 * AT_TILE * (HD * 2 + 16)];  // K then V rows of a tile (row stride padded by 16 bytes)
  float sq[GQ * HD];
  float sp[GQ][AT_TILE];
  float s_m[GQ], s_l[GQ], s_f[GQ];
  float cw[GQ][AT_MAX_SPLITS], cl[GQ][AT_MAX_SPLITS], cL[GQ];
  int s_last;
};

// group barrier: the whole CTA (BAR 0) or named barrier BAR of AT_THREADS threads.  The id is an
// immediate so that the compiler reserves every barrier the kernel uses.
template <int BAR>
__device__ __forceinline__ void attn_sync() {
  if constexpr (BAR == 0) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(AT_THREADS) : "memory");
  }
}

// One (kv head, split) work item.  tid: thread index within the group of AT_THREADS.
template <int HD, int GQ, bool MEGA, int BAR>
__device__ __forceinline__ void attn_body(const gsdlq_attn_job_t& J, int layer, int kvh, int split, int nsplit, int tps,
                                          int tid, AttnSmem<HD, GQ>& S, const unsigned* dep, unsigned dep_target,
                                          unsigned* done, unsigned* abort) {
  constexpr int ROWB = HD * 2 + 16;         // padded row bytes
  constexpr int CH = HD / 8;                // 16-byte chunks per row
  constexpr int DP = HD / 2;                // dimension pairs
  constexpr int HS = AT_THREADS / DP;       // token groups of the P.V mapping
  constexpr int NO = (GQ * HD + AT_THREADS - 1) / AT_THREADS;  // outputs per thread
  constexpr int CQ = CH / 4;                // 16-byte chunks of a K row per score thread
  // Chunk of a K row that score thread quarter qd reads at step cc.  The 8 threads of a
  // quarter-warp phase are two tokens (rows 16 bytes apart modulo 128) x four quarters; this
  // order puts the four quarters 32 bytes apart, so the 8 reads cover 8 different 16-byte bank
  // groups (no conflict).  Every quarter still covers CQ distinct chunks and all quarters all CH.
  auto kchunk = [](int qd, int cc) -> int {
    if constexpr (CQ == 4) return 2 * qd + 8 * (cc & 1) + (cc >> 1);
    else if constexpr (CQ == 2) return 2 * qd + cc;
    else return qd * CQ + cc;
  };
  uint8_t* skv = S.skv;
  uint8_t* sk = skv;
  uint8_t* sv = skv + AT_TILE * ROWB;
  float* sq = S.sq;
  auto& sp = S.sp;
  float* s_m = S.s_m;
  float* s_l = S.s_l;
  float* s_f = S.s_f;
  const int lane = tid & 31, warp = tid >> 5;
  if (!MEGA) pdl_trigger_ops();  // the next launch may be scheduled at once (its wait covers this grid)
  const int pos = J.pos_dev ? *J.pos_dev : J.pos_val;
  const bool pos_ok = pos >= 0 && pos < J.max_seq;
  const int len = pos_ok ? pos + 1 : 0;
  const int t0 = split * tps, t1 = min(len, t0 + tps);
  const size_t tok_stride = (size_t)J.n_kv_heads * HD;
  auto row_off = [&](int t) -> size_t {
    const size_t slot = J.block_table ? (size_t)J.block_table[t / J.page_size] * J.page_size + (t % J.page_size)
                                      : (size_t)layer * J.max_seq + t;
    return slot * tok_stride + (size_t)kvh * HD;
  };
  // asynchronous copies of the rows of [tb, tb + nt) selected by `which` (0: < pos, 1: == pos, 2: all)
  auto issue = [&](int tb, int nt, int which) {
    for (int i = tid; i < nt * CH; i += AT_THREADS) {
      const int j = i / CH, c = i - j * CH, t = tb + j;
      if (which == 2 || (which == 0 ? t < pos : t == pos)) {
        const size_t off = row_off(t) + c * 8;
        cp_async_16(sk + j * ROWB + c * 16, J.k_cache + off);
        cp_async_16(sv + j * ROWB + c * 16, J.v_cache + off);
      }
    }
    cp_async_commit();
  };
  if (t1 > t0) issue(t0, min(AT_TILE, t1 - t0), 0);
  if (J.fwd_acc != nullptr) {
    // the next linear's Vt columns of this head group, for the combining CTA: each split prefetches
    // its share of the 128-byte lines into L2 (rows of fwd_k, GQ*HD fp16 columns from kvh*GQ*HD)
    const int lines_per_row = GQ * HD * 2 / 128, n_lines = J.fwd_k * lines_per_row;
    for (int i = split * AT_THREADS + tid; i < n_lines; i += nsplit * AT_THREADS) {
      const int j = i / lines_per_row, c = i - j * lines_per_row;
      const uint8_t* a = reinterpret_cast<const uint8_t*>(J.fwd_vt + (size_t)j * J.n_heads * HD + (size_t)kvh * GQ * HD) + c * 128;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
    }
  }
  if (MEGA) {
    if (tid == 0 && dep != nullptr) wait_geq_abort(dep, dep_target, abort);
    attn_sync<BAR>();
  } else {
    pdl_wait_ops();
  }
  if (!pos_ok && tid == 0 && kvh == 0 && split == 0) raise_flag(GSDLQ_FLAG_BAD_POS);
  if (t1 > t0) issue(t0, min(AT_TILE, t1 - t0), 1);
  // q is staged with its 8-float chunks permuted: slot 4 * cc + qd holds the chunk that score
  // thread quarter qd takes at step cc (kchunk), so the four quarters' reads of one step fall in
  // four different bank groups.  (.cg: in the decode kernel q was written earlier in the launch.)
  for (int i = tid; i < GQ * HD; i += AT_THREADS) {
    const int h = i / HD, r = i - h * HD, slot = r >> 3;
    sq[i] = __ldcg(J.q + (size_t)kvh * GQ * HD + h * HD + kchunk(slot & 3, slot >> 2) * 8 + (r & 7));
  }
  if (tid < GQ) {
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.f;
  }
  // P.V state: thread -> dimension pair dp, tokens j = tg (mod HS), every head; each V element is
  // converted once
  const int dp = tid % DP, tg = tid / DP;
  float acc[GQ][2];
#pragma unroll
  for (int h = 0; h < GQ; ++h) acc[h][0] = acc[h][1] = 0.f;
  for (int tb = t0; tb < t1; tb += AT_TILE) {
    const int nt = min(AT_TILE, t1 - tb);
    cp_async_wait_all();
    attn_sync<BAR>();
    // scores: four threads per token, each a quarter of the dimensions, all heads
    {
      const int j = tid >> 2, qd = tid & 3;
      float s[GQ];
#pragma unroll
      for (int h = 0; h < GQ; ++h) s[h] = 0.f;
      if (j < nt) {
#pragma unroll
        for (int cc = 0; cc < CQ; ++cc) {
          const int c = kchunk(qd, cc);
          const uint4 kr = *reinterpret_cast<const uint4*>(sk + j * ROWB + c * 16);
          const float k0 = h2f(kr.x & 0xffffu), k1 = h2f(kr.x >> 16), k2 = h2f(kr.y & 0xffffu), k3 = h2f(kr.y >> 16);
          const float k4 = h2f(kr.z & 0xffffu), k5 = h2f(kr.z >> 16), k6 = h2f(kr.w & 0xffffu), k7 = h2f(kr.w >> 16);
#pragma unroll
          for (int h = 0; h < GQ; ++h) {
            const float4 qa = *reinterpret_cast<const float4*>(sq + h * HD + (4 * cc + qd) * 8);
            const float4 qb = *reinterpret_cast<const float4*>(sq + h * HD + (4 * cc + qd) * 8 + 4);
            s[h] = fmaf(qa.x, k0, s[h]);
            s[h] = fmaf(qa.y, k1, s[h]);
            s[h] = fmaf(qa.z, k2, s[h]);
            s[h] = fmaf(qa.w, k3, s[h]);
            s[h] = fmaf(qb.x, k4, s[h]);
            s[h] = fmaf(qb.y, k5, s[h]);
            s[h] = fmaf(qb.z, k6, s[h]);
            s[h] = fmaf(qb.w, k7, s[h]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < GQ; ++h) {
        s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);
        s[h] += __shfl_xor_sync(0xffffffffu, s[h], 2);
        if (qd == 0 && j < nt) sp[h][j] = s[h] * J.sm_scale;
      }
    }
    attn_sync<BAR>();
    // running softmax of the split: warp h handles head h (and h + 8 ... none: GQ <= 8)
    if (warp < GQ) {
      const int h = warp;
      const float a = lane < nt ? sp[h][lane] : -INFINITY;
      const float b = lane + 32 < nt ? sp[h][lane + 32] : -INFINITY;
      const float mt = warp_max(fmaxf(a, b));
      const float m_old = s_m[h];
      const float m = fmaxf(m_old, mt);
      const float ea = lane < nt ? expf(a - m) : 0.f;
      const float eb = lane + 32 < nt ? expf(b - m) : 0.f;
      if (lane < nt) sp[h][lane] = ea;
      if (lane + 32 < nt) sp[h][lane + 32] = eb;
      const float sum = warp_sum(ea + eb);
      if (lane == 0) {
        const float f = (m_old == -INFINITY) ? 0.f : expf(m_old - m);
        s_f[h] = f;
        s_m[h] = m;
        s_l[h] = s_l[h] * f + sum;
      }
    }
    attn_sync<BAR>();
    // P.V
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
      const float f = s_f[h];
      acc[h][0] *= f;
      acc[h][1] *= f;
    }
    for (int j = tg; j < nt; j += HS) {
      const uint32_t v2 = *reinterpret_cast<const uint32_t*>(sv + j * ROWB + dp * 4);
      const float v0 = h2f(v2 & 0xffffu), v1 = h2f(v2 >> 16);
#pragma unroll
      for (int h = 0; h < GQ; ++h) {
        const float p = sp[h][j];
        acc[h][0] = fmaf(p, v0, acc[h][0]);
        acc[h][1] = fmaf(p, v1, acc[h][1]);
      }
    }
    if (tb + AT_TILE < t1) {
      attn_sync<BAR>();  // every read of this tile is done before the next one is copied in
      issue(tb + AT_TILE, min(AT_TILE, t1 - tb - AT_TILE), 2);
    }
  }
  // sum the token groups (the staging buffers are free now): red[(tg * GQ + h) * HD + d]
  attn_sync<BAR>();
  float* red = reinterpret_cast<float*>(skv);
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
    red[(tg * GQ + h) * HD + 2 * dp] = acc[h][0];
    red[(tg * GQ + h) * HD + 2 * dp + 1] = acc[h][1];
  }
  attn_sync<BAR>();
  float res[NO];
#pragma unroll
  for (int k = 0; k < NO; ++k) {
    const int o = tid + k * AT_THREADS;
    res[k] = 0.f;
    if (o < GQ * HD) {
      const int h = o / HD, d = o - h * HD;
      for (int g = 0; g < HS; ++g) res[k] += red[(g * GQ + h) * HD + d];
    }
  }
  // Low-rank forwarding into the next linear (J.fwd_acc): this head group's GQ*HD outputs (ov[k] =
  // output tid + k * AT_THREADS) against columns kvh*GQ*HD + o of the next Vt rows, summed over
  // the group into one fixed-point atomic per row.  The K/V buffers are free by then.
  auto forward = [&](const float (&ov)[NO]) {
    if (J.fwd_acc == nullptr) return;  // uniform
    float* fr = reinterpret_cast<float*>(skv);  // [AT_THREADS / 32][fwd_k]
    const int nk = J.fwd_k;
    const int n_in = J.n_heads * HD;  // the next linear's columns
    for (int j0 = 0; j0 < nk; j0 += 16) {
      uint16_t vv[16][NO];  // every load of the block in flight at once
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const uint16_t* vt = J.fwd_vt + (size_t)(j0 + jj) * n_in + (size_t)kvh * GQ * HD;
#pragma unroll
        for (int k = 0; k < NO; ++k) {
          const int o = tid + k * AT_THREADS;
          vv[jj][k] = (j0 + jj < nk && o < GQ * HD) ? __ldg(vt + o) : (uint16_t)0;
        }
      }
      float pj[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < NO; ++k) a = fmaf(h2f(vv[jj][k]), ov[k], a);
        pj[jj] = warp_sum(a);
      }
      if (lane == 0) {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) fr[warp * 16 + jj] = pj[jj];
      }
      attn_sync<BAR>();
      if (tid < 16 && j0 + tid < nk) {
        float a = 0.f;
        for (int w = 0; w < AT_THREADS / 32; ++w) a += fr[w * 16 + tid];
        if (!(fabsf(a) < 4194304.f)) {
          raise_flag(GSDLQ_FLAG_RANGE);
          a = (a != a) ? 0.f : copysignf(4194304.f, a);
        }
        atomicAdd(J.fwd_acc + j0 + tid, (unsigned long long)__float2ll_rn(a * 4294967296.f));
      }
      attn_sync<BAR>();
    }
  };
  const int nact = min(nsplit, (len + tps - 1) / tps);
  if (nact == 1) {
    // a single split holds the whole sequence: write the output directly
    if (split == 0) {
      float ov[NO];
#pragma unroll
      for (int k = 0; k < NO; ++k) {
        const int o = tid + k * AT_THREADS;
        ov[k] = 0.f;
        if (o < GQ * HD) {
          const float l = s_l[o / HD];
          ov[k] = l > 0.f ? res[k] / l : 0.f;
          J.out[(size_t)kvh * GQ * HD + o] = ov[k];
        }
      }
      attn_sync<BAR>();  // (the K/V buffers held the token-group reduction until here)
      forward(ov);
    }
    if (MEGA && split == 0) {  // publish the head to the next phase
      __threadfence();
      attn_sync<BAR>();
      if (tid == 0) red_add_release(done, 1u);
    }
    return;
  }
  float* part = J.partial + ((size_t)kvh * nsplit + split) * (size_t)GQ * (HD + 2);
#pragma unroll
  for (int k = 0; k < NO; ++k) {
    const int o = tid + k * AT_THREADS;
    if (o < GQ * HD) part[(o / HD) * (HD + 2) + (o % HD)] = res[k];
  }
  if (tid < GQ) {
    const bool any = t1 > t0;
    part[tid * (HD + 2) + HD] = any ? s_m[tid] : -INFINITY;
    part[tid * (HD + 2) + HD + 1] = any ? s_l[tid] : 0.f;
  }
  // the last CTA of this kv head combines all splits
  __threadfence();
  attn_sync<BAR>();
  if (tid == 0) S.s_last = (atomicAdd(&J.workspace[kvh], 1u) == (unsigned)nsplit - 1);
  attn_sync<BAR>();
  if (!S.s_last) return;
  __threadfence();
  const float* base = J.partial + (size_t)kvh * nsplit * GQ * (HD + 2);
  // one batch of loads: every split's (max, sum) and this thread's partial values
  auto& cw = S.cw;
  auto& cl = S.cl;
  float* cL = S.cL;
  float mv = -INFINITY, lv = 0.f;
  const int gi = tid / nact, si = tid - gi * nact;
  if (tid < GQ * nact) {
    const float* ps = base + ((size_t)si * GQ + gi) * (HD + 2);
    mv = __ldcg(ps + HD);
    lv = __ldcg(ps + HD + 1);
  }
  constexpr int NB = NO < 2 ? NO : 2;  // outputs whose partials are loaded with the maxima
  float pv[NB][AT_MAX_SPLITS];
  auto load_pv = [&](int k0) {
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int o = tid + (k0 + k) * AT_THREADS;
      const int g = o / HD, d = o - g * HD;
#pragma unroll
      for (int sidx = 0; sidx < AT_MAX_SPLITS; ++sidx)
        pv[k][sidx] = (k0 + k < NO && o < GQ * HD && sidx < nact) ? __ldcg(base + ((size_t)sidx * GQ + g) * (HD + 2) + d) : 0.f;
    }
  };
  load_pv(0);
  if (tid < GQ * nact) {
    cw[gi][si] = mv;
    cl[gi][si] = lv;
  }
  attn_sync<BAR>();
  if (warp < GQ) {  // warp g: head g, lane = split (AT_MAX_SPLITS <= 32)
    const int g = warp;
    const float ms = lane < nact ? cw[g][lane] : -INFINITY;
    const float M = warp_max(ms);
    const float f = (ms == -INFINITY) ? 0.f : expf(ms - M);
    const float L = warp_sum(lane < nact ? cl[g][lane] * f : 0.f);
    if (lane < nact) cw[g][lane] = f;
    if (lane == 0) cL[g] = L;
  }
  attn_sync<BAR>();
  float ov[NO];
#pragma unroll
  for (int k = 0; k < NO; ++k) ov[k] = 0.f;
  for (int k0 = 0; k0 < NO; k0 += NB) {
    if (k0 > 0) load_pv(k0);
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int o = tid + (k0 + k) * AT_THREADS;
      if (k0 + k < NO && o < GQ * HD) {
        const int g = o / HD;
        float a = 0.f;
#pragma unroll
        for (int sidx = 0; sidx < AT_MAX_SPLITS; ++sidx)
          if (sidx < nact) a += pv[k][sidx] * cw[g][sidx];
        const float L = cL[g];
        const float r = (L > 0.f) ? a / L : 0.f;
        J.out[(size_t)kvh * GQ * HD + o] = r;
#pragma unroll
        for (int kk = 0; kk < NO; ++kk)
          if (kk == k0 + k) ov[kk] = r;
      }
    }
  }
  forward(ov);
  if (tid == 0) J.workspace[kvh] = 0u;
  if (MEGA) {  // publish the head to the next phase
    __threadfence();
    attn_sync<BAR>();
    if (tid == 0) red_add_release(done, 1u);
  }
}

// the P.V token-group reduction reuses the K/V staging buffers; shapes where it does not fit are
// not instantiated (head_dim 32 with more than 5 query heads per kv head)
template <int HD, int GQ>
constexpr bool attn_fits() {
  return (AT_THREADS / (HD / 2)) * GQ * HD * 4 <= 2 * AT_TILE * (HD * 2 + 16);
}


template <int HD, int GQ>
__global__ void __launch_bounds__(AT_THREADS, 2) attn_kernel(const __grid_constant__ gsdlq_attn_job_t J, int tps) {
  __shared__ AttnSmem<HD, GQ> S;
  attn_body<HD, GQ, false, 0>(J, J.layer, blockIdx.x, blockIdx.y, gridDim.y, tps, threadIdx.x, S, nullptr, 0u,
                              nullptr, nullptr);
}

}  // namespace gsdlq

// common.cuh -- shared device helpers for the GSD-LQ sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "gsdlq.h"  // include/ is on the include path

namespace gsdlq {

constexpr int kWarp = 32;

// Device-side error word.  Kernels never trap: on a violated precondition they
// skip the offending access and OR a bit in here; the host reads it with
// gsdlq_device_flags().
extern __device__ unsigned int g_device_flags;

__device__ __forceinline__ void raise_flag(unsigned int bit) { atomicOr(&g_device_flags, bit); }

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }

// bf16 bits (high half of an fp32) <-> float
__device__ __forceinline__ float bf16lo_to_f(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi_to_f(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Pack (a, b) -> bf16x2 with a in the low half, round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// Split (a, b) into hi + lo bf16x2 parts: a ~= hi.x + lo.x to about 16 mantissa bits.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(a, b);
  const float ra = a - bf16lo_to_f(hi);
  const float rb = b - bf16hi_to_f(hi);
  lo = pack_bf16x2(ra, rb);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 8-byte global load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

// 16-byte streaming load; the L2 fetches the whole 256-byte sector group around it (a unit reads
// 256 contiguous bytes of a row in four steps)
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t smem_addr) {
  uint32_t r;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(r) : "r"(smem_addr));
  return r;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Asynchronous global -> shared copies (no register staging, no load/store ordering stalls).
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, fp32 accumulate.  Not volatile: a pure
// function of its operands, so the compiler may interleave independent MMAs and loads.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                               const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

// Bounded spin on a global counter until it EQUALS `target`: returns false (and raises a
// flag) when that did not happen within ~`max_ns` nanoseconds of %globaltimer.  Equality
// rather than >= makes a counter that did not start at zero (a dirty workspace) show up as
// a timeout instead of an early, silent read.
__device__ __forceinline__ bool wait_counter_eq(const unsigned int* ctr, unsigned int target,
                                                unsigned long long max_ns) {
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr));
    if (v == target) return true;
    unsigned long long t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > max_ns) {
      raise_flag(GSDLQ_FLAG_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
}

__device__ __forceinline__ void red_add_release(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded spin until *ctr >= target (acquire), for the persistent decode kernel's phase
// dependencies.  Gives up after 1 s of %globaltimer, or at once when *abort is set: on giving
// up it raises GSDLQ_FLAG_TIMEOUT and sets *abort, so that every later wait of the launch
// returns at once and the kernel ends with the flag raised instead of hanging.
// Each poll is one load: the abort word is read only every 32nd poll (it matters only once some
// wait has already given up), and there is no sleep between polls.
__device__ __forceinline__ void wait_geq_abort(const unsigned* ctr, unsigned target, unsigned* abort) {
  unsigned long long t0 = 0ull;
  for (int it = 0;; ++it) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return;
    if ((it & 31) == 31 && *reinterpret_cast<volatile unsigned*>(abort) != 0u) return;
    unsigned long long t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (it == 0) t0 = t1;
    if (t1 - t0 > 1000000000ull) {
      raise_flag(GSDLQ_FLAG_TIMEOUT);
      atomicExch(abort, 1u);
      return;
    }
  }
}

// wait_counter_eq (1 s bound) that also returns at once when *abort (if given) is set, and sets it
// when it gives up
__device__ __forceinline__ void wait_eq_abort(const unsigned* ctr, unsigned target, unsigned* abort) {
  if (abort == nullptr) {
    wait_counter_eq(ctr, target, 1000000000ull);
    return;
  }
  unsigned long long t0 = 0ull;
  for (int it = 0;; ++it) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v == target) return;
    if (*reinterpret_cast<volatile unsigned*>(abort) != 0u) return;
    unsigned long long t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (it == 0) t0 = t1;
    if (t1 - t0 > 1000000000ull) {
      raise_flag(GSDLQ_FLAG_TIMEOUT);
      atomicExch(abort, 1u);
      return;
    }
    __nanosleep(64);
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// ---- mbarrier + TMA (bulk tensor copies into this CTA's own shared memory) -------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// make initialised barriers visible to the asynchronous (TMA) proxy
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// arrive once and add `bytes` to the transaction count of the current phase
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0u;
}
// Bounded wait for the phase of `bar` with the given parity: false (flag raised) after 1 s.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0, t1;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (!mbar_try_wait(bar, parity)) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > 1000000000ull) {
      raise_flag(GSDLQ_FLAG_TIMEOUT);
      return false;
    }
  }
  return true;
}
// 2-D tiled copy of one box at element coordinates (x, y) of `tmap` (a tensor map in parameter,
// constant or global memory) into shared memory at `dst`, completing on `bar`.  x * element size
// must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Bulk prefetch of `bytes` (a multiple of 16) at a 16-byte aligned global address into the L2 cache.
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// CTA `cta` of `n_cta` issues its share of a launch's L2 prefetch list with the 32 lanes of one
// warp: range r is cut into n_cta equal 16-byte-aligned slices and this CTA's slice into 16 KB bulk
// prefetches dealt round-robin to the lanes.  (The host checked the alignment and n <= 16.)
__device__ __forceinline__ void issue_prefetch(const gsdlq_prefetch_t& pf, unsigned cta, unsigned n_cta, int lane) {
  const int n = pf.n < GSDLQ_MAX_PREFETCH ? pf.n : GSDLQ_MAX_PREFETCH;
  constexpr unsigned long long CHUNK = 1024;  // 16-byte units per bulk prefetch
  for (int r = 0; r < n; ++r) {
    const unsigned long long units = pf.bytes[r] >> 4;
    const unsigned long long u0 = units * cta / n_cta, u1 = units * (cta + 1) / n_cta;
    const char* base = static_cast<const char*>(pf.ptr[r]);
    for (unsigned long long u = u0 + (unsigned long long)lane * CHUNK; u < u1; u += 32 * CHUNK) {
      const unsigned long long e = u + CHUNK < u1 ? u + CHUNK : u1;
      l2_prefetch_bulk(base + u * 16, (uint32_t)((e - u) * 16));
    }
  }
}

// Host check of a prefetch list: n in [0, GSDLQ_MAX_PREFETCH], 16-byte aligned ranges.
inline bool prefetch_ok(const gsdlq_prefetch_t& pf) {
  if (pf.n < 0 || pf.n > GSDLQ_MAX_PREFETCH) return false;
  for (int r = 0; r < pf.n; ++r) {
    if ((pf.bytes[r] & 15u) != 0u) return false;
    if (pf.bytes[r] != 0u && (pf.ptr[r] == nullptr || (reinterpret_cast<uintptr_t>(pf.ptr[r]) & 15u) != 0u)) return false;
  }
  return true;
}

// ---- phase trace (compiled in only with -DGSDLQ_TRACE; a diagnostic build, not the product) ----
// Each CTA of a stand-alone fused-linear launch stamps %globaltimer at fixed points of its run into
// g_trace[launch][cta][point]; launch = how many launches this CTA index has started since the last
// reset.  Read back with gsdlq_trace_read (defined in trace builds only).
#ifdef GSDLQ_TRACE
constexpr int TR_CTAS = 160, TR_LAUNCHES = 192, TR_POINTS = 32;
extern __device__ unsigned long long g_trace[TR_LAUNCHES * TR_CTAS * TR_POINTS];
extern __device__ unsigned g_trace_cnt[TR_CTAS];
__device__ __forceinline__ unsigned long long tr_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long* tr_rec(unsigned slot) {
  return g_trace + ((size_t)slot * TR_CTAS + blockIdx.x) * TR_POINTS;
}
#define GSDLQ_TR_SET(slot, pt, v)                                               \
  do {                                                                          \
    if ((slot) < (unsigned)TR_LAUNCHES && blockIdx.x < (unsigned)TR_CTAS) tr_rec(slot)[pt] = (v); \
  } while (0)
#define GSDLQ_TR_MAX(slot, pt)                                                  \
  do {                                                                          \
    if ((slot) < (unsigned)TR_LAUNCHES && blockIdx.x < (unsigned)TR_CTAS) atomicMax(tr_rec(slot) + (pt), tr_now()); \
  } while (0)
#else
#define GSDLQ_TR_SET(slot, pt, v) \
  do {                            \
  } while (0)
#define GSDLQ_TR_MAX(slot, pt) \
  do {                         \
  } while (0)
#endif

// Monotone float -> uint32 map (larger float -> larger key).
__device__ __forceinline__ uint32_t ordered_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// The reference's nan_to_num before argmax (gsd_lq_cpu_runtime.py:423).
__device__ __forceinline__ float sanitize_logit(float v) {
  if (isnan(v)) return -1e4f;
  if (isinf(v)) return v > 0.f ? 100.f : -1e4f;
  return v;
}

// 64-bit argmax key: larger value wins, then the LOWER index wins.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  return (static_cast<unsigned long long>(ordered_key(sanitize_logit(v))) << 32) |
         static_cast<unsigned long long>(0xffffffffu - idx);
}

}  // namespace gsdlq

#define GSDLQ_CUDA_CHECK_LAUNCH()                               \
  do {                                                          \
    cudaError_t _e = cudaGetLastError();                        \
    if (_e != cudaSuccess) return gsdlq::record_cuda_error(_e); \
  } while (0)

namespace gsdlq {
int record_cuda_error(cudaError_t e);
int num_sms();
}  // namespace gsdlq

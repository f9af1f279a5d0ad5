// comm.cuh -- the tensor-parallel exchange buffer shared by the all-reduce kernels (comm.cu) and the
// fused linear's exchange epilogue (hexmv_dev.cuh): its descriptor and the low-latency slot helpers.
//
// A slot is 8 bytes: 4 bytes of data (fp32 bits, or one half of a 64-bit key) and the 4-byte call
// number of the exchange that wrote it.  An aligned 8-byte store is single-copy atomic, so a reader
// that sees the current call number in a slot also sees that call's data: no fence and no separate
// flag are needed.  Slots are double-buffered by the parity of the call number.
#pragma once
#include "common.cuh"

namespace gsdlq {

constexpr int CM_CHUNK = 1024;    // elements per CTA of the all-reduce kernel
constexpr int CM_THREADS = 256;   // 4 elements per thread
constexpr int CM_MAX_WORLD = 8;

// Layout of one rank's exchange buffer (offsets in bytes from its base):
//   [0, off_keys)        u64 data[2][W][n_chunks * CM_CHUNK]   all-reduce kernel slots
//   [off_keys, ...)      u64 keys[2][W][2]                     argmax-key slots
//   [off_count, ...)     u32 count[n_chunks + 1]               completed all-reduce calls per chunk (+ key)
//   [off_excount, ...)   u32 ex[2]                             completed epilogue exchanges, CTA arrivals
//   [off_exdata, ...)    u64 exdata[2][W][n_max]               fused-epilogue exchange slots
struct CommDesc {
  uint8_t* base[CM_MAX_WORLD];  // every rank's exchange buffer (this rank's own at [rank])
  int world, rank, n_max, n_chunks;
  size_t off_keys, off_count, off_excount, off_exdata;
};

// The descriptor of a connected exchange (host; GSDLQ_ERR_INVALID if it is not connected).
int comm_desc(const gsdlq_comm_t* comm, CommDesc* out);

__device__ __forceinline__ void st_vol_v2(unsigned long long* p, unsigned long long a, unsigned long long b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void st_vol_u64(unsigned long long* p, unsigned long long a) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ void ld_vol_v2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned long long ld_vol_u64(const unsigned long long* p) {
  unsigned long long a;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}
__device__ __forceinline__ unsigned long long ll_pack(float v, unsigned k) {
  return (unsigned long long)__float_as_uint(v) | ((unsigned long long)k << 32);
}

// ---- fused-epilogue exchange ---------------------------------------------------------------------
// slot of (call k, source rank src, row) in rank `owner`'s buffer
__device__ __forceinline__ unsigned long long* ex_slot(const CommDesc& d, int owner, unsigned k, int src, int row) {
  return reinterpret_cast<unsigned long long*>(d.base[owner] + d.off_exdata) +
         ((size_t)(k & 1u) * d.world + src) * d.n_max + row;
}
__device__ __forceinline__ unsigned* ex_words(const CommDesc& d) {
  return reinterpret_cast<unsigned*>(d.base[d.rank] + d.off_excount);
}
// Wait (bounded by `deadline`, a %globaltimer value set on first use) until this rank's slot of
// (k, src, row) holds call k, and return its value; on giving up GSDLQ_FLAG_TIMEOUT is raised once.
// Polls sleep briefly between reads, so that thousands of waiting threads do not flood the L2 that
// the peers' stores land in.
__device__ __forceinline__ float ex_wait(const CommDesc& d, unsigned k, int src, int row, unsigned long long& deadline,
                                         bool& gave_up) {
  const unsigned long long* p = ex_slot(d, d.rank, k, src, row);
  for (;;) {
    const unsigned long long v = ld_vol_u64(p);
    if ((unsigned)(v >> 32) == k || gave_up) return __uint_as_float((unsigned)v);
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (deadline == 0ull) deadline = t + 1000000000ull;
    if (t > deadline) {
      raise_flag(GSDLQ_FLAG_TIMEOUT);
      gave_up = true;
    }
    __nanosleep(128);
  }
}

}  // namespace gsdlq

// comm.cu -- the tensor-parallel exchange: a one-shot all-reduce among the ranks of one node over
// peer memory (CUDA IPC mappings of each rank's exchange buffer, NVLink stores).
//
// Low-latency slots: every 8-byte store carries 4 bytes of data and a 4-byte call number, so a
// receiver knows a slot is filled when it reads the current call number in it -- no fence and no
// separate flag round trip.  (An aligned 8-byte store is single-copy atomic: the receiver never sees
// a new call number beside an old value.)  Every rank owns one exchange buffer in its own memory:
//
//   u64  data[2][W][N]   slot (call parity, source rank, element): value bits | call << 32
//   u64  keys[2][W][2]   the same for the two halves of a 64-bit argmax key
//   u32  count[NC + 1]   this rank's completed calls per chunk (and of the key reduction)
//
// A call of the all-reduce sum on x[n] runs one CTA per 1024-element chunk.  CTA c of rank s, on its
// k-th call (k = count[c] + 1, the same on every rank because every rank makes the same calls):
//   1. waits for the producer of x (programmatic dependent launch) and reads its chunk of x;
//   2. stores (x[i] | k << 32) into data[k & 1][s][i] of every OTHER rank's buffer;
//   3. polls its own data[k & 1][r][i] of every other rank r until the call number there is k
//      (bounded by 1 s of %globaltimer, after which GSDLQ_FLAG_TIMEOUT is raised and it goes on);
//   4. writes x[i] = sum over r = 0..W-1 of x_r[i] in rank order (its own value at r = s), so that
//      every rank holds the same bits; 5. sets count[c] = k.
// Two parities suffice: a rank starts call k + 2 only after its call k + 1 received every peer's
// values, which every peer sends only after it has finished reading call k.  The argmax reduction is
// the same protocol on the two halves of one 64-bit key, taking the maximum.
//
// No TMA, no multicast: plain stores to peer memory and volatile loads of this rank's own memory.
#include <cstring>

#include "comm.cuh"

namespace gsdlq {

struct gsdlq_comm_impl {  // behind the opaque gsdlq_comm_t
  CommDesc d;
  void* local = nullptr;
  size_t bytes = 0;
  int device = 0;
};

inline size_t cm_align(size_t v) { return (v + 255) & ~size_t(255); }

static void cm_layout(CommDesc& d) {
  d.n_chunks = (d.n_max + CM_CHUNK - 1) / CM_CHUNK;
  const size_t data = sizeof(unsigned long long) * 2 * (size_t)d.world * (size_t)d.n_chunks * CM_CHUNK;
  d.off_keys = cm_align(data);
  d.off_count = cm_align(d.off_keys + sizeof(unsigned long long) * 2 * 2 * d.world);
  d.off_excount = cm_align(d.off_count + sizeof(unsigned) * (d.n_chunks + 1));
  d.off_exdata = cm_align(d.off_excount + 2 * sizeof(unsigned));
}

static size_t cm_bytes(const CommDesc& d) {
  return cm_align(d.off_exdata + sizeof(unsigned long long) * 2 * (size_t)d.world * (size_t)d.n_max);
}

// Poll the two slots at p (this rank's memory) until both carry call number k; bounded by `deadline`
// (a %globaltimer value, 0 = not started): on giving up it raises GSDLQ_FLAG_TIMEOUT once and
// returns whatever the slots hold.
__device__ __forceinline__ void ll_wait2(const unsigned long long* p, unsigned k, unsigned long long& a,
                                         unsigned long long& b, unsigned long long& deadline, bool& gave_up) {
  for (;;) {
    ld_vol_v2(p, a, b);
    if ((unsigned)(a >> 32) == k && (unsigned)(b >> 32) == k) return;
    if (gave_up) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (deadline == 0ull) deadline = t + 1000000000ull;
    if (t > deadline) {
      raise_flag(GSDLQ_FLAG_TIMEOUT);
      gave_up = true;
      return;
    }
  }
}

__global__ void __launch_bounds__(CM_THREADS) comm_allreduce_sum_kernel(const __grid_constant__ CommDesc d, float* x,
                                                                       int n) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x is complete once the previous grid has ended
  __shared__ unsigned s_k;
  const int c = blockIdx.x, tid = threadIdx.x;
  unsigned* count = reinterpret_cast<unsigned*>(d.base[d.rank] + d.off_count) + c;
  if (tid == 0) s_k = *reinterpret_cast<volatile unsigned*>(count) + 1u;
  __syncthreads();
  const unsigned k = s_k;
  const size_t stride_src = (size_t)d.n_chunks * CM_CHUNK;
  const size_t par_off = (size_t)(k & 1u) * d.world * stride_src;
  const int i0 = c * CM_CHUNK + tid * 4;  // (the slots cover whole chunks: no tail guard on them)
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = (i0 + j < n) ? __ldcg(x + i0 + j) : 0.f;
  // 2. this rank's values into every other rank's slots
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank) continue;
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(d.base[r]) + par_off + (size_t)d.rank * stride_src + i0;
    st_vol_v2(dst, ll_pack(v[0], k), ll_pack(v[1], k));
    st_vol_v2(dst + 2, ll_pack(v[2], k), ll_pack(v[3], k));
  }
  // 3. + 4. every other rank's values, summed in rank order
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  unsigned long long deadline = 0ull;
  bool gave_up = false;
  for (int r = 0; r < d.world; ++r) {
    float t[4];
    if (r == d.rank) {
#pragma unroll
      for (int j = 0; j < 4; ++j) t[j] = v[j];
    } else {
      const unsigned long long* src =
          reinterpret_cast<const unsigned long long*>(d.base[d.rank]) + par_off + (size_t)r * stride_src + i0;
      unsigned long long a, b, e, f;
      ll_wait2(src, k, a, b, deadline, gave_up);
      ll_wait2(src + 2, k, e, f, deadline, gave_up);
      t[0] = __uint_as_float((unsigned)a), t[1] = __uint_as_float((unsigned)b);
      t[2] = __uint_as_float((unsigned)e), t[3] = __uint_as_float((unsigned)f);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] = r == 0 ? t[j] : s[j] + t[j];
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (i0 + j < n) x[i0 + j] = s[j];
  __syncthreads();  // every thread has read k
  if (tid == 0) *reinterpret_cast<volatile unsigned*>(count) = k;
}

__global__ void comm_allreduce_max_u64_kernel(const __grid_constant__ CommDesc d, unsigned long long* key) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x != 0) return;
  unsigned* count = reinterpret_cast<unsigned*>(d.base[d.rank] + d.off_count) + d.n_chunks;
  const unsigned k = *reinterpret_cast<volatile unsigned*>(count) + 1u;
  const size_t par_off = (size_t)(k & 1u) * d.world * 2;
  const unsigned long long v = *reinterpret_cast<volatile unsigned long long*>(key);
  const unsigned long long lo = (v & 0xffffffffull) | ((unsigned long long)k << 32);
  const unsigned long long hi = (v >> 32) | ((unsigned long long)k << 32);
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank) continue;
    st_vol_v2(reinterpret_cast<unsigned long long*>(d.base[r] + d.off_keys) + par_off + 2 * d.rank, lo, hi);
  }
  unsigned long long m = v, deadline = 0ull;
  bool gave_up = false;
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank) continue;
    unsigned long long a, b;
    ll_wait2(reinterpret_cast<const unsigned long long*>(d.base[d.rank] + d.off_keys) + par_off + 2 * r, k, a, b,
             deadline, gave_up);
    const unsigned long long t = (a & 0xffffffffull) | (b << 32);
    m = t > m ? t : m;
  }
  *key = m;
  *reinterpret_cast<volatile unsigned*>(count) = k;
}

static int cm_launch_cfg(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, int grid, int threads, cudaStream_t s) {
  cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return GSDLQ_OK;
}

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_comm_create(int world, int rank, int n_max, gsdlq_comm_t** comm, void* ipc_handle) {
  if (!comm || !ipc_handle || world < 1 || world > CM_MAX_WORLD || rank < 0 || rank >= world || n_max <= 0)
    return GSDLQ_ERR_INVALID;
  *comm = nullptr;
  gsdlq_comm_impl* c = new gsdlq_comm_impl();
  c->d.world = world;
  c->d.rank = rank;
  c->d.n_max = n_max;
  cm_layout(c->d);
  c->bytes = cm_bytes(c->d);
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->local, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return record_cuda_error(e);
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == GSDLQ_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle, &h, sizeof(h));
  for (int r = 0; r < CM_MAX_WORLD; ++r) c->d.base[r] = nullptr;
  c->d.base[rank] = static_cast<uint8_t*>(c->local);
  *comm = reinterpret_cast<gsdlq_comm_t*>(c);
  return GSDLQ_OK;
}

extern "C" int gsdlq_comm_connect(gsdlq_comm_t* comm, const void* handles) {
  gsdlq_comm_impl* c = reinterpret_cast<gsdlq_comm_impl*>(comm);
  if (!c || !handles) return GSDLQ_ERR_INVALID;
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < c->d.world; ++r) {
    if (r == c->d.rank || c->d.base[r] != nullptr) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + (size_t)r * GSDLQ_IPC_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return record_cuda_error(e);
    c->d.base[r] = static_cast<uint8_t*>(p);
  }
  return GSDLQ_OK;
}

namespace gsdlq {
int comm_desc(const gsdlq_comm_t* comm, CommDesc* out) {
  const gsdlq_comm_impl* c = reinterpret_cast<const gsdlq_comm_impl*>(comm);
  if (!c || !out) return GSDLQ_ERR_INVALID;
  for (int r = 0; r < c->d.world; ++r)
    if (c->d.base[r] == nullptr) return GSDLQ_ERR_INVALID;
  *out = c->d;
  return GSDLQ_OK;
}
}  // namespace gsdlq

static bool cm_ready(const gsdlq_comm_impl* c) {
  for (int r = 0; r < c->d.world; ++r)
    if (c->d.base[r] == nullptr) return false;
  return true;
}

extern "C" int gsdlq_comm_allreduce_sum(gsdlq_comm_t* comm, float* x, int n, gsdlq_stream_t stream) {
  gsdlq_comm_impl* c = reinterpret_cast<gsdlq_comm_impl*>(comm);
  if (!c || !x || n <= 0 || n > c->d.n_max || (reinterpret_cast<uintptr_t>(x) & 15u)) return GSDLQ_ERR_INVALID;
  if (!cm_ready(c)) return GSDLQ_ERR_INVALID;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  // every rank runs all n_chunks CTAs (the per-chunk call counts stay equal across ranks and calls)
  cm_launch_cfg(cfg, attr, c->d.n_chunks, CM_THREADS, static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaLaunchKernelEx(&cfg, comm_allreduce_sum_kernel, c->d, x, n);
  return e == cudaSuccess ? GSDLQ_OK : record_cuda_error(e);
}

extern "C" int gsdlq_comm_allreduce_max_u64(gsdlq_comm_t* comm, unsigned long long* key, gsdlq_stream_t stream) {
  gsdlq_comm_impl* c = reinterpret_cast<gsdlq_comm_impl*>(comm);
  if (!c || !key || (reinterpret_cast<uintptr_t>(key) & 7u)) return GSDLQ_ERR_INVALID;
  if (!cm_ready(c)) return GSDLQ_ERR_INVALID;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  cm_launch_cfg(cfg, attr, 1, 32, static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaLaunchKernelEx(&cfg, comm_allreduce_max_u64_kernel, c->d, key);
  return e == cudaSuccess ? GSDLQ_OK : record_cuda_error(e);
}

extern "C" int gsdlq_comm_destroy(gsdlq_comm_t* comm) {
  gsdlq_comm_impl* c = reinterpret_cast<gsdlq_comm_impl*>(comm);
  if (!c) return GSDLQ_OK;
  int status = GSDLQ_OK;
  for (int r = 0; r < c->d.world; ++r) {
    if (r == c->d.rank || c->d.base[r] == nullptr) continue;
    const cudaError_t e = cudaIpcCloseMemHandle(c->d.base[r]);
    if (e != cudaSuccess) status = record_cuda_error(e);
  }
  if (c->local) {
    const cudaError_t e = cudaFree(c->local);
    if (e != cudaSuccess) status = record_cuda_error(e);
  }
  delete c;
  return status;
}

// ops.cu -- the non-GEMV kernels of the engine and the C-ABI glue.
//
//   rmsnorm / vec_add / swiglu / lowrank_proj   drop-ins for gsd_lq_cpu_engine.c:67-127
//   rope_and_store_kv                           drop-in for gsd_lq_cpu_engine.c:186-262
//   attention (split-KV decode)                 gsd_lq_cpu_engine.c:265-330, engine + drop-in
//   dequant                                     gsd_lq_cpu_runtime.py:281-284 (bit-exact W)
//   argmax                                      gsd_lq_cpu_runtime.py:422-425
//   pack_lattice                                the packer's lattice step (no reference counterpart)
#include <cmath>
#include <cstdio>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <vector>

#include <algorithm>

#include "common.cuh"
#include "attn_dev.cuh"
#include "attn_cluster.cuh"

namespace gsdlq {

__device__ unsigned int g_device_flags = 0;

static thread_local int t_last_cuda_error = 0;

int record_cuda_error(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return GSDLQ_ERR_CUDA;
}

int num_sms() {
  static std::atomic<int> cached[64];  // per device; racing look-ups store the same count
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// ---------------------------------------------------------------------------------------
// elementwise drop-ins
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
                               int n, float eps) {
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(t / (float)n + eps);
  }
  __syncthreads();
  const float inv = red[0];
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

__global__ void vec_add_kernel(float* y, const float* a, const float* b, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

__global__ void swiglu_kernel(const float* gate, const float* up, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float g = gate[i];
    out[i] = (g / (1.0f + expf(-g))) * up[i];
  }
}

__global__ void lowrank_kernel(const float* __restrict__ x, const uint16_t* __restrict__ vt,
                               const float* __restrict__ S, float* __restrict__ tmp_k, int cols) {
  __shared__ float red[32];
  const int j = blockIdx.x;
  const uint16_t* row = vt + (size_t)j * cols;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) s += x[c] * h2f(row[c]);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    tmp_k[j] = t * S[j];
  }
}

// ---------------------------------------------------------------------------------------
// RoPE + fp16 KV store (drop-in).  The angles' cosines/sines arrive precomputed.
struct RopeParams {
  float2 cs[256];  // (cos, sin) for i < head_dim/2
};

__global__ void rope_store_kernel(float* q, const float* k, const float* v, uint16_t* kc, uint16_t* vc,
                                  size_t base, int n_heads, int n_kv, int hd, int interleaved,
                                  const __grid_constant__ RopeParams rp) {
  const int half = hd / 2;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int nq = n_heads * half, nk = n_kv * half;
  if (t < nq) {
    const int h = t / half, i = t - h * half;
    const int i0 = interleaved ? 2 * i : i, i1 = interleaved ? 2 * i + 1 : i + half;
    float* qh = q + (size_t)h * hd;
    const float a = qh[i0], b = qh[i1];
    const float c = rp.cs[i].x, s = rp.cs[i].y;
    qh[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    qh[i1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  } else if (t < nq + nk) {
    const int u = t - nq;
    const int h = u / half, i = u - h * half;
    const int i0 = interleaved ? 2 * i : i, i1 = interleaved ? 2 * i + 1 : i + half;
    const float* kh = k + (size_t)h * hd;
    const float a = kh[i0], b = kh[i1];
    const float c = rp.cs[i].x, s = rp.cs[i].y;
    kc[base + (size_t)h * hd + i0] = f2h(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)));
    kc[base + (size_t)h * hd + i1] = f2h(__fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c)));
    const float* vh = v + (size_t)h * hd;
    vc[base + (size_t)h * hd + i0] = f2h(vh[i0]);
    vc[base + (size_t)h * hd + i1] = f2h(vh[i1]);
  }
}

template <int HD, int GQ>
static cudaError_t attention_launch_t(const cudaLaunchConfig_t& cfg, const gsdlq_attn_job_t& J, int tps) {
  if constexpr (attn_fits<HD, GQ>()) return cudaLaunchKernelEx(&cfg, attn_kernel<HD, GQ>, J, tps);
  return cudaErrorNotSupported;
}

template <int HD>
static cudaError_t attention_launch_hd(const cudaLaunchConfig_t& cfg, const gsdlq_attn_job_t& J, int tps, int gq) {
  switch (gq) {
    case 1: return attention_launch_t<HD, 1>(cfg, J, tps);
    case 2: return attention_launch_t<HD, 2>(cfg, J, tps);
    case 3: return attention_launch_t<HD, 3>(cfg, J, tps);
    case 4: return attention_launch_t<HD, 4>(cfg, J, tps);
    case 5: return attention_launch_t<HD, 5>(cfg, J, tps);
    case 6: return attention_launch_t<HD, 6>(cfg, J, tps);
    case 7: return attention_launch_t<HD, 7>(cfg, J, tps);
    default: return attention_launch_t<HD, 8>(cfg, J, tps);
  }
}

// The cluster kernel (attn_cluster.cuh) serves every stand-alone launch unless GSDLQ_ATTN_CLUSTER=0
// (read once per process) selects the split/counter kernel (attn_kernel).
static bool attn_cluster_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GSDLQ_ATTN_CLUSTER");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <int HD, int GQ>
static cudaError_t attention_cluster_launch_t(const gsdlq_attn_job_t& J, cudaStream_t s) {
  using Lo = AcLayout<HD, GQ>;
  if constexpr (Lo::BYTES > 227 * 1024) {
    return cudaErrorNotSupported;
  } else {
    static std::atomic<bool> smem_set[64];  // per device: the dynamic shared-memory opt-in is done
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64) return cudaErrorNotSupported;
    if (!smem_set[dev].load(std::memory_order_acquire)) {
      e = cudaFuncSetAttribute(attn_cluster_kernel<HD, GQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, Lo::BYTES);
      if (e != cudaSuccess) return e;
      smem_set[dev].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(AC_CL, J.n_kv_heads);
    cfg.blockDim = dim3(AC_THREADS);
    cfg.dynamicSmemBytes = Lo::BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = AC_CL;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, attn_cluster_kernel<HD, GQ>, J);
  }
}

template <int HD>
static cudaError_t attention_cluster_launch_hd(const gsdlq_attn_job_t& J, cudaStream_t s, int gq) {
  switch (gq) {
    case 1: return attention_cluster_launch_t<HD, 1>(J, s);
    case 2: return attention_cluster_launch_t<HD, 2>(J, s);
    case 3: return attention_cluster_launch_t<HD, 3>(J, s);
    case 4: return attention_cluster_launch_t<HD, 4>(J, s);
    case 5: return attention_cluster_launch_t<HD, 5>(J, s);
    case 6: return attention_cluster_launch_t<HD, 6>(J, s);
    case 7: return attention_cluster_launch_t<HD, 7>(J, s);
    default: return attention_cluster_launch_t<HD, 8>(J, s);
  }
}

static int attention_launch(const gsdlq_attn_job_t& J, cudaStream_t s) {
  if (!J.q || !J.k_cache || !J.v_cache || !J.out || !J.partial || !J.workspace) return GSDLQ_ERR_INVALID;
  // K/V rows are read in 16-byte chunks
  if ((reinterpret_cast<uintptr_t>(J.k_cache) | reinterpret_cast<uintptr_t>(J.v_cache)) & 15u) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(J.q) & 3u) return GSDLQ_ERR_INVALID;
  if (J.n_heads <= 0 || J.n_kv_heads <= 0 || J.n_heads % J.n_kv_heads) return GSDLQ_ERR_INVALID;
  const int gq = J.n_heads / J.n_kv_heads;
  if (gq > AT_MAX_GQ) return GSDLQ_ERR_UNSUPPORTED;
  if (J.max_seq <= 0 || J.layer < 0) return GSDLQ_ERR_INVALID;
  if (J.block_table && J.page_size <= 0) return GSDLQ_ERR_INVALID;
  if (!J.pos_dev && (J.pos_val < 0 || J.pos_val >= J.max_seq)) return GSDLQ_ERR_INVALID;
  if (J.fwd_acc && (J.fwd_k <= 0 || J.fwd_k > 48 || !J.fwd_vt || (reinterpret_cast<uintptr_t>(J.fwd_acc) & 7u)))
    return GSDLQ_ERR_INVALID;
  if (J.head_dim != 128 && J.head_dim != 64 && J.head_dim != 32) return GSDLQ_ERR_UNSUPPORTED;
  if (!prefetch_ok(J.prefetch)) return GSDLQ_ERR_INVALID;  // (only the cluster kernel issues it)
  // the cluster kernel copies the forwarded Vt slice in 4-byte pieces
  if (attn_cluster_enabled() && !(J.fwd_acc && (reinterpret_cast<uintptr_t>(J.fwd_vt) & 3u))) {
    cudaError_t e;
    if (J.head_dim == 128) e = attention_cluster_launch_hd<128>(J, s, gq);
    else if (J.head_dim == 64) e = attention_cluster_launch_hd<64>(J, s, gq);
    else e = attention_cluster_launch_hd<32>(J, s, gq);
    if (e == cudaSuccess) return GSDLQ_OK;
    if (e != cudaErrorNotSupported) return record_cuda_error(e);
  }
  const int tps = attn_tokens_per_split(J.max_seq);
  const int nsplit = (J.max_seq + tps - 1) / tps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(J.n_kv_heads, nsplit);
  cfg.blockDim = dim3(AT_THREADS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (J.head_dim == 128) e = attention_launch_hd<128>(cfg, J, tps, gq);
  else if (J.head_dim == 64) e = attention_launch_hd<64>(cfg, J, tps, gq);
  else if (J.head_dim == 32) e = attention_launch_hd<32>(cfg, J, tps, gq);
  else return GSDLQ_ERR_UNSUPPORTED;
  if (e == cudaErrorNotSupported) return GSDLQ_ERR_UNSUPPORTED;
  if (e != cudaSuccess) return record_cuda_error(e);
  return GSDLQ_OK;
}

static void attention_ws(int n_heads, int n_kv, int hd, int max_seq, size_t* pb, size_t* wb) {
  const int tps = attn_tokens_per_split(max_seq);
  const int ns = (max_seq + tps - 1) / tps;
  *pb = sizeof(float) * (size_t)n_kv * ns * (n_heads / n_kv) * (hd + 2);
  *wb = sizeof(unsigned) * (size_t)n_kv;
}

// scratch for the drop-in gsdlq_gqa_attention (whose signature carries none):
// allocated on the first call per device and grown on demand.
struct DropinScratch {
  float* partial = nullptr;
  unsigned* ws = nullptr;
  size_t pbytes = 0, wbytes = 0;
};
static std::mutex g_scratch_mu;
static DropinScratch g_scratch[64];

// ---------------------------------------------------------------------------------------
__global__ void dequant_kernel(const uint8_t* __restrict__ codes, const uint16_t* __restrict__ scales,
                               const float* __restrict__ xy, float* __restrict__ w, size_t n, int n_pts) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int c = codes[i >> 1];
    float t = 0.f;
    if (c < n_pts) t = xy[2 * c + (i & 1)];
    else raise_flag(GSDLQ_FLAG_BAD_CODE);
    w[i] = __fmul_rn(t, h2f(scales[i >> 6]));
  }
}

__global__ void argmax_kernel(const float* __restrict__ x, int n, int* out) {
  __shared__ unsigned long long red[32];
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long k = argmax_key(x[i], (uint32_t)i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = red[w] > b ? red[w] : b;
    *out = (int)(0xffffffffu - (uint32_t)(b & 0xffffffffull));
  }
}

// Lattice step of the packer; one warp per (row, 64-column group), lane = pair.
// float32 arithmetic without contraction, mirroring gsdlq_b200.packer.quantize_lattice.
__constant__ unsigned char c_code_index[2][17 * 17];  // [radius==8][(r0+R)*(2R+1) + r1+R] -> code, 255 outside
__constant__ signed char c_coords[2][217 * 2];        // code -> (r0, r1)
__constant__ float c_xy[2][217 * 2];                  // code -> float32 lattice point (the reference table)

__global__ void pack_lattice_kernel(const float* __restrict__ w, int rows, int cols, int radius, int rsel,
                                    uint8_t* __restrict__ codes, uint16_t* __restrict__ scales,
                                    float* __restrict__ resid) {
  const int lane = threadIdx.x & 31;
  const size_t gid = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const size_t G = cols / 64;
  if (gid >= (size_t)rows * G) return;
  const size_t e0 = gid * 64 + 2 * lane;  // element index of this lane's pair (groups never straddle rows)
  const float w0 = w[e0], w1 = w[e0 + 1];
  float amax = fmaxf(fabsf(w0), fabsf(w1));
  amax = warp_max(amax);
  const float FIT = 0.6339746117591858f;  // float32(1/(1+1/sqrt(3)))
  const float H = 0.8660253882408142f;    // float32(sqrt(3)/2)
  const float IH = 1.1547005176544189f;   // float32(2/sqrt(3))
  const float sc = __fdiv_rn(amax, __fmul_rn((float)radius, FIT));
  const uint16_t sbits = f2h(sc);
  const float s32 = h2f(sbits);
  const float inv = (s32 > 0.f) ? __fdiv_rn(1.0f, s32) : 0.f;
  const float u = __fmul_rn(w0, inv), v = __fmul_rn(w1, inv);
  const float r1f = __fmul_rn(v, IH);
  const float r0f = __fsub_rn(u, __fmul_rn(0.5f, r1f));
  const int a = (int)floorf(r0f), b = (int)floorf(r1f);
  float bd = 0.f;
  int b0 = 0, b1 = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c0 = a + (k & 1), c1 = b + (k >> 1);
    const float px = __fadd_rn((float)c0, __fmul_rn(0.5f, (float)c1));
    const float py = __fmul_rn((float)c1, H);
    const float dx = __fsub_rn(u, px), dy = __fsub_rn(v, py);
    const float d = __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
    if (k == 0 || d < bd) { bd = d; b0 = c0; b1 = c1; }
  }
  const int R = radius;
  const int n_pts = (R == 8) ? 217 : 127;
  int code;
  // written so that garbage from non-finite inputs (floorf of NaN/inf) also takes the exhaustive path
  const bool inside = b0 >= -R && b0 <= R && b1 >= -R && b1 <= R && b0 + b1 >= -R && b0 + b1 <= R;
  if (!inside) {
    // nearest hexagon point by exhaustive search, first minimum wins (np.argmin)
    float best = 0.f;
    code = 0;
    for (int i = 0; i < n_pts; ++i) {
      const float q0 = (float)c_coords[rsel][2 * i], q1 = (float)c_coords[rsel][2 * i + 1];
      const float qx = __fadd_rn(q0, __fmul_rn(0.5f, q1));
      const float qy = __fmul_rn(q1, H);
      const float dx = __fsub_rn(u, qx), dy = __fsub_rn(v, qy);
      const float d = __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
      if (i == 0 || d < best) { best = d; code = i; }
    }
  } else {
    code = c_code_index[rsel][(b0 + R) * (2 * R + 1) + (b1 + R)];
  }
  codes[e0 >> 1] = (uint8_t)code;
  if (lane == 0) scales[gid] = sbits;
  if (resid) {
    resid[e0] = __fsub_rn(w0, __fmul_rn(c_xy[rsel][2 * code], s32));
    resid[e0 + 1] = __fsub_rn(w1, __fmul_rn(c_xy[rsel][2 * code + 1], s32));
  }
}

__global__ void greedy_advance_kernel(unsigned long long* key, int* token, int* pos, int* step, int* out_ids,
                                      int max_out) {
  const unsigned long long k = *key;
  const int t = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
  *token = t;
  if (out_ids != nullptr && *step < max_out) out_ids[*step] = t;
  *step += 1;
  *pos += 1;
  *key = 0ull;
}

// gsdlq_greedy_advance with the reference chat loop's EOS stop (run_gpu_native_chat.py:1142-1144): once
// the picked token is eos_id, *done is set and nothing more advances (the EOS token is not stored)
__global__ void advance_eos_kernel(unsigned long long* key, int* token, int* pos, int* step, int* out_ids, int max_out,
                                   int eos_id, int* done) {
  if (*done) {
    *key = 0ull;
    return;
  }
  const unsigned long long k = *key;
  const int t = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
  *key = 0ull;
  if (t == eos_id) {
    *done = 1;
    return;
  }
  *token = t;
  if (out_ids != nullptr && *step < max_out) out_ids[*step] = t;
  *step += 1;
  *pos += 1;
}

static int host_codebook(int radius, float* xy, int max_pts) {
  if (radius < 1 || radius > 8) return GSDLQ_ERR_INVALID;
  const double h = std::sqrt(3.0) / 2.0;
  int n = 0;
  for (int r0 = -radius; r0 <= radius; ++r0)
    for (int r1 = -radius; r1 <= radius; ++r1) {
      if (std::abs(r0 + r1) > radius) continue;
      if (xy && n < max_pts) {
        xy[2 * n] = (float)((double)r0 + 0.5 * (double)r1);
        xy[2 * n + 1] = (float)((double)r1 * h);
      }
      ++n;
    }
  return n;
}

static int ensure_pack_tables() {
  static std::once_flag once;
  static int status = GSDLQ_OK;
  std::call_once(once, [] {
    unsigned char idx[2][17 * 17];
    signed char crd[2][217 * 2] = {};
    float xy[2][217 * 2] = {};
    for (int s = 0; s < 2; ++s) {
      const int R = s ? 8 : 6;
      for (int i = 0; i < 17 * 17; ++i) idx[s][i] = 255;
      host_codebook(R, xy[s], 217);
      int c = 0;
      for (int r0 = -R; r0 <= R; ++r0)
        for (int r1 = -R; r1 <= R; ++r1)
          if (std::abs(r0 + r1) <= R) {
            idx[s][(r0 + R) * (2 * R + 1) + (r1 + R)] = (unsigned char)c;
            crd[s][2 * c] = (signed char)r0;
            crd[s][2 * c + 1] = (signed char)r1;
            ++c;
          }
    }
    cudaError_t e = cudaMemcpyToSymbol(c_code_index, idx, sizeof(idx));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_coords, crd, sizeof(crd));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_xy, xy, sizeof(xy));
    if (e != cudaSuccess) status = record_cuda_error(e);
  });
  return status;
}

}  // namespace gsdlq

using namespace gsdlq;

// ======================================================================================
extern "C" {

const char* gsdlq_status_string(int st) {
  switch (st) {
    case GSDLQ_OK: return "ok";
    case GSDLQ_ERR_INVALID: return "invalid argument";
    case GSDLQ_ERR_CUDA: return "CUDA error";
    case GSDLQ_ERR_UNSUPPORTED: return "unsupported configuration";
    default: return "unknown status";
  }
}

int gsdlq_last_cuda_error(void) { return t_last_cuda_error; }

const char* gsdlq_version(void) { return "0.1.0 sm_100a"; }

int gsdlq_device_flags(unsigned int* flags, gsdlq_stream_t stream) {
  if (!flags) return GSDLQ_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(flags, g_device_flags, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_device_flags, &zero, sizeof(unsigned), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? GSDLQ_OK : record_cuda_error(e);
}

int gsdlq_rmsnorm(const float* x, const float* weight, float* out, int dim, float eps, gsdlq_stream_t stream) {
  if (!x || !weight || !out || dim <= 0) return GSDLQ_ERR_INVALID;
  rmsnorm_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, weight, out, dim, eps);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_vec_add(float* y, const float* a, const float* b, int dim, gsdlq_stream_t stream) {
  if (!y || !a || !b || dim <= 0) return GSDLQ_ERR_INVALID;
  vec_add_kernel<<<(dim + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, a, b, dim);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_swiglu(const float* gate, const float* up, float* out, int dim, gsdlq_stream_t stream) {
  if (!gate || !up || !out || dim <= 0) return GSDLQ_ERR_INVALID;
  swiglu_kernel<<<(dim + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(gate, up, out, dim);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_lowrank_proj(const float* x, const uint16_t* Vt, const float* S, float* tmp_k, int k_dim, int cols,
                       gsdlq_stream_t stream) {
  if (k_dim == 0) return GSDLQ_OK;
  if (!x || !Vt || !S || !tmp_k || k_dim < 0 || k_dim > 16 || cols <= 0) return GSDLQ_ERR_INVALID;
  lowrank_kernel<<<k_dim, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, Vt, S, tmp_k, cols);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_rope_table(float* table, int max_seq, int head_dim, float rope_theta) {
  if (!table || max_seq <= 0 || head_dim <= 0 || head_dim % 2) return GSDLQ_ERR_INVALID;
  const int half = head_dim / 2;
  for (int p = 0; p < max_seq; ++p)
    for (int i = 0; i < half; ++i) {
      // gsd_lq_cpu_engine.c:215-218, evaluated with the host C library as the reference does
      const float freq = 1.0f / powf(rope_theta, (float)(2 * i) / (float)head_dim);
      const float ang = (float)p * freq;
      table[((size_t)p * half + i) * 2] = cosf(ang);
      table[((size_t)p * half + i) * 2 + 1] = sinf(ang);
    }
  return GSDLQ_OK;
}

int gsdlq_rope_and_store_kv(float* q, const float* k, const float* v, uint16_t* k_cache, uint16_t* v_cache,
                            int layer_idx, int pos, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
                            float rope_theta, int interleaved, gsdlq_stream_t stream) {
  if (!q || !k || !v || !k_cache || !v_cache) return GSDLQ_ERR_INVALID;
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 || head_dim > 512) return GSDLQ_ERR_INVALID;
  if (pos < 0 || pos >= max_seq_len || layer_idx < 0) return GSDLQ_ERR_INVALID;
  RopeParams rp;
  const int half = head_dim / 2;
  for (int i = 0; i < half; ++i) {
    const float freq = 1.0f / powf(rope_theta, (float)(2 * i) / (float)head_dim);
    const float ang = (float)pos * freq;
    rp.cs[i] = make_float2(cosf(ang), sinf(ang));
  }
  const size_t base = (size_t)layer_idx * max_seq_len * n_kv_heads * head_dim + (size_t)pos * n_kv_heads * head_dim;
  const int n = (n_heads + n_kv_heads) * half;
  rope_store_kernel<<<(n + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, k_cache, v_cache, base, n_heads, n_kv_heads, head_dim, interleaved ? 1 : 0, rp);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_attention_ws_size(int n_heads, int n_kv_heads, int head_dim, int max_seq, size_t* partial_bytes,
                            size_t* workspace_bytes) {
  if (!partial_bytes || !workspace_bytes || n_kv_heads <= 0 || n_heads % n_kv_heads || max_seq <= 0)
    return GSDLQ_ERR_INVALID;
  attention_ws(n_heads, n_kv_heads, head_dim, max_seq, partial_bytes, workspace_bytes);
  return GSDLQ_OK;
}

int gsdlq_attention(const gsdlq_attn_job_t* job, gsdlq_stream_t stream) {
  if (!job) return GSDLQ_ERR_INVALID;
  return attention_launch(*job, static_cast<cudaStream_t>(stream));
}

int gsdlq_gqa_attention(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, float* attn_out,
                        int layer_idx, int pos, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
                        float sm_scale, gsdlq_stream_t stream) {
  if (n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads || max_seq_len <= 0) return GSDLQ_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u) return GSDLQ_ERR_INVALID;
  size_t pb = 0, wb = 0;
  attention_ws(n_heads, n_kv_heads, head_dim, max_seq_len, &pb, &wb);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e);
  if (dev < 0 || dev >= 64) return GSDLQ_ERR_UNSUPPORTED;
  DropinScratch* sc = &g_scratch[dev];
  // held through the launch: another thread's grow frees the buffers this launch is given
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  {
    if (sc->pbytes < pb) {
      if (sc->partial) cudaFree(sc->partial);
      sc->partial = nullptr;
      sc->pbytes = 0;
      e = cudaMalloc(&sc->partial, pb);
      if (e != cudaSuccess) return record_cuda_error(e);
      sc->pbytes = pb;
    }
    if (sc->wbytes < wb) {
      if (sc->ws) cudaFree(sc->ws);
      sc->ws = nullptr;
      sc->wbytes = 0;
      e = cudaMalloc(&sc->ws, wb);
      if (e != cudaSuccess) return record_cuda_error(e);
      e = cudaMemset(sc->ws, 0, wb);
      if (e != cudaSuccess) return record_cuda_error(e);
      sc->wbytes = wb;
    }
  }
  gsdlq_attn_job_t J{};
  J.q = q;
  J.k_cache = k_cache;
  J.v_cache = v_cache;
  J.out = attn_out;
  J.pos_dev = nullptr;
  J.pos_val = pos;
  J.layer = layer_idx;
  J.n_heads = n_heads;
  J.n_kv_heads = n_kv_heads;
  J.head_dim = head_dim;
  J.max_seq = max_seq_len;
  J.sm_scale = sm_scale;
  J.partial = sc->partial;
  J.workspace = sc->ws;
  return attention_launch(J, static_cast<cudaStream_t>(stream));
}

int gsdlq_codebook(int radius, float* xy_out, int max_pts) { return host_codebook(radius, xy_out, max_pts); }

int gsdlq_dequant(const uint8_t* codes, const uint16_t* scales, const float* xy_table, float* w, int rows, int cols,
                  int n_pts, gsdlq_stream_t stream) {
  if (!codes || !scales || !xy_table || !w || rows <= 0 || cols <= 0 || cols % 64 || n_pts <= 0 || n_pts > 256)
    return GSDLQ_ERR_INVALID;
  const size_t n = (size_t)rows * cols;
  const int grid = (int)std::min<size_t>((n + 255) / 256, (size_t)num_sms() * 16);
  dequant_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(codes, scales, xy_table, w, n, n_pts);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_argmax(const float* logits, int n, int* out_index, gsdlq_stream_t stream) {
  if (!logits || !out_index || n <= 0) return GSDLQ_ERR_INVALID;
  argmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(logits, n, out_index);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_advance_eos(unsigned long long* argmax_key, int* token, int* pos, int* step, int* out_ids, int max_out,
                      int eos_id, int* done, gsdlq_stream_t stream) {
  if (!argmax_key || !token || !pos || !step || !done) return GSDLQ_ERR_INVALID;
  advance_eos_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(argmax_key, token, pos, step, out_ids, max_out,
                                                                     eos_id, done);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_greedy_advance(unsigned long long* argmax_key, int* token, int* pos, int* step, int* out_ids, int max_out,
                         gsdlq_stream_t stream) {
  if (!argmax_key || !token || !pos || !step) return GSDLQ_ERR_INVALID;
  greedy_advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(argmax_key, token, pos, step, out_ids, max_out);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

int gsdlq_pack_lattice(const float* w, int rows, int cols, int radius, uint8_t* codes, uint16_t* scales,
                       float* residual, gsdlq_stream_t stream) {
  if (!w || !codes || !scales || rows <= 0 || cols <= 0 || cols % 64) return GSDLQ_ERR_INVALID;
  if (radius != 6 && radius != 8) return GSDLQ_ERR_INVALID;
  const int st = ensure_pack_tables();
  if (st != GSDLQ_OK) return st;
  const size_t groups = (size_t)rows * (cols / 64);
  const size_t threads = groups * 32;
  const unsigned grid = (unsigned)((threads + 255) / 256);
  pack_lattice_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(w, rows, cols, radius, radius == 8 ? 1 : 0,
                                                                            codes, scales, residual);
  GSDLQ_CUDA_CHECK_LAUNCH();
  return GSDLQ_OK;
}

}  // extern "C"

// hexmv.cu -- launches of the fused GSD-LQ packed linear (device code in hexmv_dev.cuh) and
// its C-ABI entry points.
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "hexmv_dev.cuh"

namespace gsdlq {

// ---- TMA descriptors -------------------------------------------------------------------------
// cuTensorMapEncodeTiled is a driver API entry point; it is looked up once through the runtime so
// that the library needs no link-time dependency on the driver library.
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Descriptors of one matrix for the TMA ring: codes [rows][cols/2] u8 in 64 x 16 boxes, scales
// [rows][cols/64] fp16 in 8 x 16 boxes.  Rows past the end read as zero.
int hexmv_encode_maps(const gsdlq_hexmat_t& M, CUtensorMap* codes, CUtensorMap* scales) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
  if (enc == nullptr) return GSDLQ_ERR_UNSUPPORTED;
  const cuuint64_t np = (cuuint64_t)M.cols / 2, g = (cuuint64_t)M.cols / 64, rows = (cuuint64_t)M.rows;
  const cuuint32_t one[2] = {1, 1};
  {
    const cuuint64_t dims[2] = {np, rows};
    const cuuint64_t strides[1] = {np};
    const cuuint32_t box[2] = {64, 16};
    if (enc(codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(M.codes), dims, strides, box, one,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GSDLQ_ERR_UNSUPPORTED;
  }
  {
    const cuuint64_t dims[2] = {g, rows};
    const cuuint64_t strides[1] = {g * 2};
    const cuuint32_t box[2] = {8, 16};
    if (enc(scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(M.scales), dims, strides, box, one,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GSDLQ_ERR_UNSUPPORTED;
  }
  return GSDLQ_OK;
}

// ---- host side ------------------------------------------------------------------------
static int hexmv_validate_mat(const gsdlq_hexmat_t& M, int cols, bool own_lowrank) {
  if (!M.codes || !M.scales || !M.row_ptr) return GSDLQ_ERR_INVALID;
  // codes are read 16 bytes at a time from row starts (cols/2 is a multiple of 32)
  if (reinterpret_cast<uintptr_t>(M.codes) & 15u) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(M.scales) & 1u) return GSDLQ_ERR_INVALID;
  if (M.rows <= 0 || M.cols != cols || cols <= 0 || cols % 64 != 0) return GSDLQ_ERR_INVALID;
  if (M.k_dim < 0 || M.k_dim > 16) return GSDLQ_ERR_INVALID;
  if (M.k_dim > 0 && !M.U) return GSDLQ_ERR_INVALID;
  if (own_lowrank && M.k_dim > 0 && (!M.S || !M.Vt)) return GSDLQ_ERR_INVALID;
  if (own_lowrank && M.k_dim > 0 && (reinterpret_cast<uintptr_t>(M.Vt) & 15u)) return GSDLQ_ERR_INVALID;  // 16-byte loads
  if (M.radius != 6 && M.radius != 8) return GSDLQ_ERR_INVALID;
  return GSDLQ_OK;
}

// In-loop L2 prefetch distance of the streaming warps, in units (GSDLQ_PF_AHEAD, default 0).
static int hexmv_pf_ahead() {
  static const int d = [] {
    const char* e = std::getenv("GSDLQ_PF_AHEAD");
    const int v = e ? std::atoi(e) : 0;
    return v < 0 ? 0 : (v > 16 ? 16 : v);
  }();
  return d;
}

// Geometry of a launch (everything but the workspace pointers).
int hexmv_plan(HexmvParams& P) {
  const gsdlq_linear_job_t& J = P.job;
  if (J.n_mat < 1 || J.n_mat > 3) return GSDLQ_ERR_INVALID;
  const int C = J.mat[0].cols;
  for (int m = 0; m < J.n_mat; ++m) {
    const int st = hexmv_validate_mat(J.mat[m], C, P.tmp_k_ext == nullptr);
    if (st != GSDLQ_OK) return st;
    if (J.mat[m].radius != J.mat[0].radius) return GSDLQ_ERR_INVALID;
  }
  P.cols = C;
  P.G = C / 64;
  P.NP = C / 2;
  P.nmat = (J.epilogue == GSDLQ_EPI_SWIGLU) ? 2 : 1;
  if (P.nmat == 2) {
    if (J.n_mat != 2) return GSDLQ_ERR_INVALID;
    P.n_strips = (J.mat[0].rows + 15) / 16;
  } else {
    P.strip_begin[0] = 0;
    for (int m = 0; m < J.n_mat; ++m) P.strip_begin[m + 1] = P.strip_begin[m] + (J.mat[m].rows + 15) / 16;
    P.n_strips = P.strip_begin[J.n_mat];
  }
  P.GU = (P.G + 7) / 8;
  P.UPS = P.nmat * P.GU;
  P.T = (long long)P.n_strips * P.UPS;
  if (P.T >= (1LL << 31)) return GSDLQ_ERR_UNSUPPORTED;  // unit indices are 32-bit in the kernel
  // one CTA per SM (fewer when there are fewer units); a range of ceil(T / n_cta) units touches at
  // most ceil(that / UPS) + 1 strips, the rows of each CTA's shared-memory accumulator
  // at least ceil(UPS / 6) units a CTA, so that a strip spans at most 7 CTAs (the shared-strip
  // words count up to 7 contributions)
  const long long upc_min = (P.UPS + 5) / 6;
  P.n_cta = (int)std::max<long long>(1, std::min<long long>(num_sms(), P.T / upc_min));
  const long long upc = (P.T + P.n_cta - 1) / P.n_cta;
  P.n_local = (int)((upc + P.UPS - 1) / P.UPS) + 1;
  const int grid = P.n_cta;
  int lr = 0;
  for (int m = 0; m < 4; ++m) P.lr_off[m] = 0;
  for (int m = 0; m < J.n_mat; ++m) {
    P.lr_off[m] = lr;
    lr += J.mat[m].k_dim;
  }
  P.n_lr = P.tmp_k_ext ? 0 : lr;
  const int helpers = grid * HX_HELP;
  P.lr_chunks = (C / 8 + helpers - 1) / helpers;
  P.ovf_bytes = std::max(0, P.GU * 16 - 256) * 128;
  // per-unit kink lists are used when every matrix has them (8-byte entries)
  P.pf_ahead = hexmv_pf_ahead();
  P.ukink = 1;
  for (int m = 0; m < J.n_mat; ++m) {
    const gsdlq_hexmat_t& M = J.mat[m];
    if (!M.unit_kink_off || !M.unit_kinks || (reinterpret_cast<uintptr_t>(M.unit_kinks) & 7u)) P.ukink = 0;
  }
  // shared-memory limits: the accumulator (16 KB), and the table region, the activation-split
  // overflow chunks and the accumulator together
  if (hx_lacc_bytes(P) > 16 * 1024 || hx_dyn_smem(P.ovf_bytes) + hx_lacc_bytes(P) > 227 * 1024)
    return GSDLQ_ERR_UNSUPPORTED;
  P.lacc_off = 0x10000 + P.ovf_bytes;  // (after the TMA ring when a launch uses it)
  return GSDLQ_OK;
}

// 16-byte scale loads: every row's scales start 16-byte aligned and no unit is partial
bool hexmv_full(const HexmvParams& P) {
  if (P.G % 8 != 0) return false;
  for (int m = 0; m < P.job.n_mat; ++m)
    if (reinterpret_cast<uintptr_t>(P.job.mat[m].scales) & 15u) return false;
  return true;
}

template <int EPI, bool FULL, bool TMA, bool UK>
static int hexmv_launch_t(const HexmvParams& P, const HxMaps& T, cudaStream_t s) {
  const int dyn = (TMA ? hx_dyn_smem_tma(P.ovf_bytes) : hx_dyn_smem(P.ovf_bytes)) + hx_lacc_bytes(P);
  static std::atomic<bool> configured[64];  // per device: the dynamic shared-memory opt-in is done
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(hexmv_kernel<EPI, FULL, TMA, UK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return record_cuda_error(e);
    configured[dev].store(true, std::memory_order_release);
  }
  const int grid = P.n_cta;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(HX_THREADS);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, hexmv_kernel<EPI, FULL, TMA, UK>, P, T);
  if (e != cudaSuccess) return record_cuda_error(e);
  return GSDLQ_OK;
}

// low-rank forwarding: a single-output epilogue, whole strips, at most 48 accumulators (the
// control block's), aligned Vt rows of the next linear
static int hexmv_check_fwd(const HexmvParams& P) {
  const gsdlq_linear_job_t& J = P.job;
  if (J.lr_forwarded && P.tmp_k_ext != nullptr) return GSDLQ_ERR_INVALID;
  if (J.fwd_acc == nullptr) return GSDLQ_OK;
  if (reinterpret_cast<uintptr_t>(J.fwd_acc) & 7u) return GSDLQ_ERR_INVALID;
  const bool single = J.epilogue == GSDLQ_EPI_RESID || J.epilogue == GSDLQ_EPI_SWIGLU ||
                      (J.epilogue == GSDLQ_EPI_STORE && J.n_mat == 1);
  if (!single || J.mat[0].rows % 16 != 0) return GSDLQ_ERR_INVALID;
  int nk = 0;
  for (int m = 0; m < 3; ++m) {
    if (J.fwd_k[m] < 0 || J.fwd_k[m] > 16) return GSDLQ_ERR_INVALID;
    if (J.fwd_k[m] > 0 && (!J.fwd_vt[m] || (reinterpret_cast<uintptr_t>(J.fwd_vt[m]) & 15u))) return GSDLQ_ERR_INVALID;
    nk += J.fwd_k[m];
  }
  return nk > 0 ? GSDLQ_OK : GSDLQ_ERR_INVALID;
}

int hexmv_check_io(const HexmvParams& P) {
  const gsdlq_linear_job_t& J = P.job;
  if (hexmv_check_fwd(P) != GSDLQ_OK) return GSDLQ_ERR_INVALID;
  if (!prefetch_ok(J.prefetch)) return GSDLQ_ERR_INVALID;
  if (J.exchange) {  // the fused tensor-parallel sum: a RESID launch of one matrix
    CommDesc d;
    if (J.epilogue != GSDLQ_EPI_RESID || J.n_mat != 1) return GSDLQ_ERR_INVALID;
    if (comm_desc(J.exchange, &d) != GSDLQ_OK || J.mat[0].rows > d.n_max) return GSDLQ_ERR_INVALID;
  }
  if (J.input_mode < 0 || J.input_mode > 2) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_PLAIN && !J.x) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_RMSNORM && (!J.x || !J.norm_w)) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_EMBED && (!J.embed || !J.token || !J.norm_w || J.vocab <= 0)) return GSDLQ_ERR_INVALID;
  if (J.input_mode != GSDLQ_IN_EMBED && (reinterpret_cast<uintptr_t>(J.x) & 7u)) return GSDLQ_ERR_INVALID;
  if (J.input_mode != GSDLQ_IN_PLAIN && (reinterpret_cast<uintptr_t>(J.norm_w) & 7u)) return GSDLQ_ERR_INVALID;
  if (J.input_mode == GSDLQ_IN_EMBED && (reinterpret_cast<uintptr_t>(J.embed) & 3u)) return GSDLQ_ERR_INVALID;
  switch (J.epilogue) {
    case GSDLQ_EPI_STORE:
      if (J.n_mat != 1 && J.argmax_key) return GSDLQ_ERR_INVALID;
      for (int m = 0; m < J.n_mat; ++m)
        if (!J.y[m]) return GSDLQ_ERR_INVALID;
      return GSDLQ_OK;
    case GSDLQ_EPI_RESID:
      return (J.n_mat != 1 || !J.y[0] || !J.resid) ? GSDLQ_ERR_INVALID : GSDLQ_OK;
    case GSDLQ_EPI_SWIGLU:
      return (J.n_mat != 2 || !J.y[0] || J.mat[0].rows != J.mat[1].rows) ? GSDLQ_ERR_INVALID : GSDLQ_OK;
    case GSDLQ_EPI_ROPE_KV:
      if (J.n_mat != 3 || !J.y[0] || !J.k_cache || !J.v_cache || !J.pos || !J.rope_cs) return GSDLQ_ERR_INVALID;
      if (J.interleaved != 1 || J.head_dim <= 0 || J.head_dim % 16 != 0 || J.max_seq <= 0) return GSDLQ_ERR_UNSUPPORTED;
      if (J.mat[1].rows != J.mat[2].rows || J.mat[0].rows % J.head_dim || J.mat[1].rows % J.head_dim)
        return GSDLQ_ERR_INVALID;
      return GSDLQ_OK;
    default:
      return GSDLQ_ERR_INVALID;
  }
}

// The TMA ring (opt-in with GSDLQ_TMA=1): FULL streams whose shared memory (table, overflow, ring)
// fits and whose descriptors could be made.  Measured on B200 it streams slower than the per-lane
// loads (two slots per warp keep too few bytes in flight), so it is not the default.
bool hexmv_tma_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GSDLQ_TMA");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}
bool hexmv_tma_ok(const HexmvParams& P) {
  return hexmv_tma_enabled() && hexmv_full(P) && hx_dyn_smem_tma(P.ovf_bytes) + hx_lacc_bytes(P) <= 227 * 1024 &&
         tmap_encoder() != nullptr;
}

template <int EPI>
static int hexmv_dispatch_full(const HexmvParams& P, cudaStream_t s) {
  HxMaps T;
  std::memset(&T, 0, sizeof(T));
  if (hexmv_tma_ok(P)) {
    bool ok = true;
    for (int m = 0; m < P.job.n_mat && ok; ++m) ok = hexmv_encode_maps(P.job.mat[m], &T.codes[m], &T.scales[m]) == GSDLQ_OK;
    if (ok) {
      HexmvParams Q = P;
      Q.lacc_off = 0x10000 + P.ovf_bytes + HX_RING_BYTES;  // the accumulator after the ring
      return hexmv_launch_t<EPI, true, true, false>(Q, T, s);
    }
  }
  if (hexmv_full(P)) return P.ukink ? hexmv_launch_t<EPI, true, false, true>(P, T, s) : hexmv_launch_t<EPI, true, false, false>(P, T, s);
  return P.ukink ? hexmv_launch_t<EPI, false, false, true>(P, T, s) : hexmv_launch_t<EPI, false, false, false>(P, T, s);
}

static int hexmv_dispatch(const HexmvParams& P, cudaStream_t s) {
  switch (P.job.epilogue) {
    case GSDLQ_EPI_STORE: return hexmv_dispatch_full<GSDLQ_EPI_STORE>(P, s);
    case GSDLQ_EPI_RESID: return hexmv_dispatch_full<GSDLQ_EPI_RESID>(P, s);
    case GSDLQ_EPI_SWIGLU: return hexmv_dispatch_full<GSDLQ_EPI_SWIGLU>(P, s);
    default: return hexmv_dispatch_full<GSDLQ_EPI_ROPE_KV>(P, s);
  }
}

int hexmv_launch(HexmvParams& P, void* workspace, size_t ws_bytes, cudaStream_t s) {
  int st = hexmv_plan(P);
  if (st != GSDLQ_OK) return st;
  st = hexmv_check_io(P);
  if (st != GSDLQ_OK) return st;
  const size_t need = hexmv_ws_bytes_for(P.n_strips, P.nmat);
  if (!workspace || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u)) return GSDLQ_ERR_INVALID;
  P.ctl = static_cast<unsigned*>(workspace);
  P.cnt = P.ctl + CTL_WORDS;
  if (P.job.exchange) {
    st = comm_desc(P.job.exchange, &P.ex);
    if (st != GSDLQ_OK) return st;
    P.ex_on = 1;
  }
  const uintptr_t pb = reinterpret_cast<uintptr_t>(P.cnt + P.n_strips);
  P.gacc = reinterpret_cast<unsigned long long*>((pb + 15) & ~uintptr_t(15));
  return hexmv_dispatch(P, s);
}

size_t hexmv_ws_bytes(HexmvParams& P) {
  if (hexmv_plan(P) != GSDLQ_OK) return 0;
  return hexmv_ws_bytes_for(P.n_strips, P.nmat);
}

// Workspace of the drop-in gsdlq_hex2d_matvec, whose signature carries none: one buffer
// per device, allocated on first use, grown on demand, zero-initialised.
struct DropinWs {
  void* p = nullptr;
  size_t bytes = 0;
};
static DropinWs g_mv_ws[64];
static DropinWs g_wide_ws[64];  // the GEMM's work for matrices the fused kernel cannot plan
static std::mutex g_mv_mu;  // guards g_mv_ws and g_wide_ws: the grow (free + malloc) and the launch that reads it

// in hexmm.cu: the GEMM with one token, for matrices the fused kernel cannot plan
size_t hexmm_wide_work_bytes(int cols);
int hexmm_matvec_wide(const float* x, const uint8_t* codes, const uint16_t* scales, const float* xy_table,
                      const uint16_t* U, const float* tmp_k, const uint32_t* kink_row_ptr, const uint16_t* kink_cols,
                      const float* kink_deltas, float* y, void* work, int rows, int cols, int k_dim, int n_pts,
                      cudaStream_t s);

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_linear_ws_size(const gsdlq_linear_job_t* job, size_t* bytes) {
  if (!job || !bytes) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  P.job = *job;
  const size_t b = hexmv_ws_bytes(P);
  if (b == 0) return GSDLQ_ERR_INVALID;
  *bytes = b;
  return GSDLQ_OK;
}

extern "C" int gsdlq_linear(const gsdlq_linear_job_t* job, void* workspace, size_t workspace_bytes,
                            gsdlq_stream_t stream) {
  if (!job) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  P.job = *job;
  return hexmv_launch(P, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int gsdlq_hex2d_matvec(const float* x, const uint8_t* codes, const uint16_t* scales, const float* xy_table,
                                  const uint16_t* U, const float* tmp_k, const uint32_t* kink_row_ptr,
                                  const uint16_t* kink_cols, const float* kink_deltas, float* y, int rows, int cols,
                                  int k_dim, int n_pts, gsdlq_stream_t stream) {
  if (!x || !codes || !scales || !xy_table || !kink_row_ptr || !y) return GSDLQ_ERR_INVALID;
  if (n_pts <= 0 || n_pts > 256) return GSDLQ_ERR_INVALID;
  if (k_dim > 0 && (!U || !tmp_k)) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  gsdlq_linear_job_t& J = P.job;
  J.n_mat = 1;
  gsdlq_hexmat_t& M = J.mat[0];
  M.codes = codes;
  M.scales = scales;
  M.U = U;
  M.row_ptr = kink_row_ptr;
  M.kink_cols = kink_cols;
  M.kink_deltas = kink_deltas;
  M.rows = rows;
  M.cols = cols;
  M.k_dim = k_dim;
  M.radius = 8;  // unused when xy_table is given
  // the drop-in signature carries no S/Vt: the low-rank term comes from the caller's tmp_k
  M.S = nullptr;
  M.Vt = nullptr;
  J.input_mode = GSDLQ_IN_PLAIN;
  J.x = x;
  J.epilogue = GSDLQ_EPI_STORE;
  J.y[0] = y;
  P.xy_table = xy_table;
  P.n_pts = n_pts;
  P.tmp_k_ext = k_dim > 0 ? tmp_k : nullptr;
  const int st = hexmv_plan(P);
  if (st != GSDLQ_OK && st != GSDLQ_ERR_UNSUPPORTED) return st;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e);
  if (dev < 0 || dev >= 64) return GSDLQ_ERR_UNSUPPORTED;
  if (st == GSDLQ_ERR_UNSUPPORTED) {
    // beyond the fused kernel's shared memory (rows wider than GSDLQ_MATVEC_MAX_COLS, or very tall and
    // wide): the dequant-GEMM with one token, same result within the matvec tolerance
    const size_t wneed = hexmm_wide_work_bytes(cols) + 1024;
    std::lock_guard<std::mutex> lock(g_mv_mu);
    DropinWs& w = g_wide_ws[dev];
    if (w.bytes < wneed) {
      if (w.p) cudaFree(w.p);
      w.p = nullptr;
      w.bytes = 0;
      e = cudaMalloc(&w.p, wneed);
      if (e != cudaSuccess) return record_cuda_error(e);
      w.bytes = wneed;
    }
    void* wa = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(w.p) + 1023) & ~static_cast<uintptr_t>(1023));
    return hexmm_matvec_wide(x, codes, scales, xy_table, U, tmp_k, kink_row_ptr, kink_cols, kink_deltas, y, wa, rows,
                             cols, k_dim, n_pts, static_cast<cudaStream_t>(stream));
  }
  const size_t need = hexmv_ws_bytes_for(P.n_strips, P.nmat);
  std::lock_guard<std::mutex> lock(g_mv_mu);
  DropinWs& ws = g_mv_ws[dev];
  if (ws.bytes < need) {
    if (ws.p) cudaFree(ws.p);
    ws.p = nullptr;
    ws.bytes = 0;
    e = cudaMalloc(&ws.p, need);
    if (e != cudaSuccess) return record_cuda_error(e);
    e = cudaMemset(ws.p, 0, need);
    if (e != cudaSuccess) return record_cuda_error(e);
    ws.bytes = need;
  }
  return hexmv_launch(P, ws.p, ws.bytes, static_cast<cudaStream_t>(stream));
}

// ---- per-unit kink lists ------------------------------------------------------------------
// Unit (strip s, column block c) holds the kinks of rows 16s .. 16s+15 with columns in
// [512c, 512c + 512), rows then columns ascending (the CSR order within each row); a column
// past the last block (an invalid kink) is kept in the last block, where the kernel flags it.
namespace gsdlq {
__device__ __forceinline__ void unit_row_range(const uint32_t* rp, const uint16_t* kc, int row, int c, int GU,
                                               uint32_t& a, uint32_t& b) {
  const uint32_t e0 = rp[row], e1 = max(rp[row + 1], e0);
  // first kink with col >= 512c, and with col >= 512(c+1) (the last block takes the rest)
  auto lower = [&](uint32_t v) {
    uint32_t lo = e0, hi = e1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if ((uint32_t)kc[mid] < v) lo = mid + 1;
      else hi = mid;
    }
    return lo;
  };
  a = c == 0 ? e0 : lower((uint32_t)c * HX_UB * 2);
  b = c == GU - 1 ? e1 : lower((uint32_t)(c + 1) * HX_UB * 2);
}

__global__ void unit_kink_count(const uint32_t* rp, const uint16_t* kc, int rows, int GU, int n_units, uint32_t* cnt) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= n_units) return;
  const int s = u / GU, c = u - s * GU;
  uint32_t n = 0u;
  for (int r = s * 16; r < min(rows, s * 16 + 16); ++r) {
    uint32_t a, b;
    unit_row_range(rp, kc, r, c, GU, a, b);
    n += b > a ? b - a : 0u;
  }
  cnt[u] = n;
}

// exclusive prefix sum of cnt[0..n) into off[0..n] (one CTA; load-time only)
__global__ void unit_kink_scan(const uint32_t* cnt, int n, uint32_t* off) {
  __shared__ uint32_t carry;
  __shared__ uint32_t wsum[32];
  if (threadIdx.x == 0) carry = 0u;
  __syncthreads();
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    uint32_t v = i < n ? cnt[i] : 0u;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
      uint32_t t = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0u;
      for (int d = 1; d < 32; d <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, t, d);
        if (lane >= d) t += y;
      }
      wsum[lane] = t;
    }
    __syncthreads();
    const uint32_t pre = carry + (warp > 0 ? wsum[warp - 1] : 0u) + x - v;
    if (i < n) off[i] = pre;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = pre + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) off[n] = carry;
}

__global__ void unit_kink_fill(const uint32_t* rp, const uint16_t* kc, const float* kd, int rows, int GU, int n_units,
                               const uint32_t* off, uint2* ent) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= n_units) return;
  const int s = u / GU, c = u - s * GU;
  uint32_t o = off[u];
  for (int r = s * 16; r < min(rows, s * 16 + 16); ++r) {
    uint32_t a, b;
    unit_row_range(rp, kc, r, c, GU, a, b);
    for (uint32_t e = a; e < b; ++e) ent[o++] = make_uint2((uint32_t)kc[e] | ((uint32_t)(r - s * 16) << 16), __float_as_uint(kd[e]));
  }
}
}  // namespace gsdlq

extern "C" int gsdlq_unit_kinks(const uint32_t* row_ptr, const uint16_t* kink_cols, const float* kink_deltas, int rows,
                                int cols, uint32_t* unit_kink_off, uint32_t* unit_kinks, gsdlq_stream_t stream) {
  if (!row_ptr || !unit_kink_off || rows <= 0 || cols <= 0 || cols % 64 != 0) return GSDLQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(unit_kinks) & 7u) return GSDLQ_ERR_INVALID;
  const int GU = (cols / 64 + 7) / 8;
  const int n_units = ((rows + 15) / 16) * GU;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the counts go to unit_kink_off + 1 .. n (shifted), then the scan writes offsets in place
  uint32_t* cnt = unit_kink_off + 1;
  const int tb = 256, nb = (n_units + tb - 1) / tb;
  unit_kink_count<<<nb, tb, 0, s>>>(row_ptr, kink_cols, rows, GU, n_units, cnt);
  GSDLQ_CUDA_CHECK_LAUNCH();
  unit_kink_scan<<<1, 1024, 0, s>>>(cnt, n_units, unit_kink_off);
  GSDLQ_CUDA_CHECK_LAUNCH();
  if (unit_kinks && kink_cols && kink_deltas) {
    unit_kink_fill<<<nb, tb, 0, s>>>(row_ptr, kink_cols, kink_deltas, rows, GU, n_units, unit_kink_off,
                                     reinterpret_cast<uint2*>(unit_kinks));
    GSDLQ_CUDA_CHECK_LAUNCH();
  }
  return GSDLQ_OK;
}

// ---- phase trace read-back (trace builds only) -------------------------------------------------
#ifdef GSDLQ_TRACE
namespace gsdlq {
__device__ unsigned long long g_trace[TR_LAUNCHES * TR_CTAS * TR_POINTS];
__device__ unsigned g_trace_cnt[TR_CTAS];
}  // namespace gsdlq
extern "C" int gsdlq_trace_reset(void) {
  static unsigned long long zero_t[TR_LAUNCHES * TR_CTAS * TR_POINTS];
  static unsigned zero_c[TR_CTAS];
  cudaError_t e = cudaMemcpyToSymbol(g_trace, zero_t, sizeof(zero_t));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_trace_cnt, zero_c, sizeof(zero_c));
  return e == cudaSuccess ? GSDLQ_OK : record_cuda_error(e);
}
extern "C" int gsdlq_trace_read(unsigned long long* out, size_t n) {
  if (n < (size_t)TR_LAUNCHES * TR_CTAS * TR_POINTS) return GSDLQ_ERR_INVALID;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_trace, sizeof(unsigned long long) * TR_LAUNCHES * TR_CTAS * TR_POINTS);
  return e == cudaSuccess ? GSDLQ_OK : record_cuda_error(e);
}
#endif

// ---- allocation-free matvec ------------------------------------------------------------
// Scratch for gsdlq_hex2d_matvec_noalloc: a fixed array in the library's device image, so a
// call never allocates.  Host code must not pass `g_noalloc_ws` itself to a kernel (on the
// host it names a stand-in, not device memory); the device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
namespace gsdlq {
static __device__ __align__(256) unsigned char g_noalloc_ws[GSDLQ_NOALLOC_WS_BYTES];
static std::atomic<void*> g_noalloc_addr[64];  // per device; racing set-ups store the same address
static_assert(sizeof(unsigned) * CTL_WORDS + 256 + 132ull * GSDLQ_NOALLOC_MAX_STRIPS + 16 <= GSDLQ_NOALLOC_WS_BYTES,
              "GSDLQ_NOALLOC_MAX_STRIPS strips must fit the fixed scratch");
}  // namespace gsdlq

extern "C" int gsdlq_hex2d_matvec_noalloc(const float* x, const uint8_t* codes, const uint16_t* scales,
                                          const float* xy_table, const uint16_t* U, const float* tmp_k,
                                          const uint32_t* kink_row_ptr, const uint16_t* kink_cols,
                                          const float* kink_deltas, float* y, int rows, int cols, int k_dim,
                                          int n_pts, gsdlq_stream_t stream) {
  if (!x || !codes || !scales || !xy_table || !kink_row_ptr || !y) return GSDLQ_ERR_INVALID;
  if (n_pts <= 0 || n_pts > 256) return GSDLQ_ERR_INVALID;
  if (k_dim > 0 && (!U || !tmp_k)) return GSDLQ_ERR_INVALID;
  HexmvParams P{};
  gsdlq_linear_job_t& J = P.job;
  J.n_mat = 1;
  gsdlq_hexmat_t& M = J.mat[0];
  M.codes = codes;
  M.scales = scales;
  M.U = U;
  M.row_ptr = kink_row_ptr;
  M.kink_cols = kink_cols;
  M.kink_deltas = kink_deltas;
  M.rows = rows;
  M.cols = cols;
  M.k_dim = k_dim;
  M.radius = 8;  // unused when xy_table is given
  J.input_mode = GSDLQ_IN_PLAIN;
  J.x = x;
  J.epilogue = GSDLQ_EPI_STORE;
  J.y[0] = y;
  P.xy_table = xy_table;
  P.n_pts = n_pts;
  P.tmp_k_ext = k_dim > 0 ? tmp_k : nullptr;
  int st = hexmv_plan(P);
  if (st != GSDLQ_OK) return st;
  st = hexmv_check_io(P);  // every argument error is returned before the set-up and the memset
  if (st != GSDLQ_OK) return st;
  const size_t need = hexmv_ws_bytes_for(P.n_strips, P.nmat);
  if (need > (size_t)GSDLQ_NOALLOC_WS_BYTES) return GSDLQ_ERR_UNSUPPORTED;  // beyond the fixed scratch
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e);
  if (dev < 0 || dev >= 64) return GSDLQ_ERR_UNSUPPORTED;
  void* ws = g_noalloc_addr[dev].load(std::memory_order_acquire);
  if (ws == nullptr) {  // set-up, once per device (this device is current)
    e = cudaGetSymbolAddress(&ws, g_noalloc_ws);
    if (e != cudaSuccess) return record_cuda_error(e);
    g_noalloc_addr[dev].store(ws, std::memory_order_release);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the array keeps whatever the previous call left: clear the bytes this launch needs at zero
  e = cudaMemsetAsync(ws, 0, need, s);
  if (e != cudaSuccess) return record_cuda_error(e);
  return hexmv_launch(P, ws, (size_t)GSDLQ_NOALLOC_WS_BYTES, s);
}

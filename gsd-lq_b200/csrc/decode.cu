// decode.cu -- the persistent decode step: every phase of one token in ONE launch.
//
// A decode token is, per layer, five dependent phases (QKV linear with RoPE + KV append,
// attention, O linear + residual, gate/up linear + SwiGLU, down linear + residual) and then the
// LM head with the greedy argmax.  Launched as separate kernels, each phase pays a launch gap,
// the spread of its CTAs' start times, a rebuild of the decode table and the drain of the
// previous kernel; those fixed costs, not HBM bandwidth, dominated the step.  Here one
// cooperative launch of one CTA per SM runs every phase in order:
//
//   - a phase is the stand-alone kernel's body (hexmv_body / attn_body) with MEGA = true, its
//     shape record read from the kernel parameters like a stand-alone launch's;
//   - a phase waits for its producer through a completion counter in global memory (one per
//     phase): every finished strip of a linear, every combined kv head of attention and every
//     CTA that has finished reading the phase's input adds 1 (release), and the consumer's
//     first thread spins (acquire, bounded) until the producer's total is reached;
//   - the decode table is built once and kept while the lattice radius stays the same;
//   - weight loads of the next phase are issued before its dependency wait, as the stand-alone
//     kernel does before griddepcontrol.wait.
//
// Counters only grow during a step; the last CTA to finish the step runs the greedy advance
// (token, position, output id) and zeroes the counters and every phase's control words, so the
// next launch starts from zero.  Every wait gives up after 1 s and then sets an abort word that
// makes all later waits return at once: a broken dependency ends the launch with
// GSDLQ_FLAG_TIMEOUT raised instead of hanging the GPU.
#include <cstring>
#include <vector>

#include "attn_dev.cuh"
#include "hexmv_dev.cuh"

namespace gsdlq {

// Phase kinds.  Every layer has the same shapes, so the kernel parameters hold one shape record
// per kind (the compiler reads its fields as constant-bank operands, as in a stand-alone launch)
// and one record of pointers per layer.
enum MkKind { MK_QKV = 0, MK_O = 1, MK_GU = 2, MK_DN = 3, MK_HEAD = 4, MK_KINDS = 5 };
constexpr int MK_PER_LAYER = 5;   // phases per layer: QKV, attention, O, gate/up, down
constexpr int MK_MAX_LAYERS = 36; // keeps the parameter block under the 32 KB kernel-parameter limit

struct MkLayer {
  gsdlq_hexmat_t mats[7];  // q, k, v, o, gate, up, down
  const float* attn_norm;
  const float* ffn_norm;
};

struct MkParams {
  HexmvParams lin[MK_KINDS];  // shape records (the layer-specific fields come from layers[])
  int gacc_off[MK_KINDS];     // byte offset of the shared strips' fixed-point sums in a strip workspace
  gsdlq_attn_job_t attn;      // attention (its layer field is replaced per layer)
  int n_layers;
  int with_head;
  int nsplit;                 // attention splits per kv head
  unsigned* sync;             // [0] abort, [1] CTAs done with the step, [2 + p] completion of phase p
  unsigned* ctl;              // control words of every phase, CTL_WORDS each
  int ctl_words;
  int n_phases;
  uint8_t* ws[2];             // strip workspaces; consecutive linear phases alternate
  const CUtensorMap* tmaps;   // TMA descriptors (codes, scales) of layer l's matrix m at 2 * (7 l + m),
                              // the head's at 2 * 7 * n_layers (device memory)
  unsigned long long* key;    // greedy bookkeeping after the head (null: none)
  int* token;
  int* pos;
  int* step;
  int* out_ids;
  int max_out;
  MkLayer layers[MK_MAX_LAYERS];
};

// The parameter block of the step being launched.  It is copied in on the launch stream before
// every step, so a plan's launches must not overlap another plan's (one stream per device, or
// ordered streams).  Each phase is a separate (not inlined) function that reads it at a fixed
// address: the compiler treats its fields as constant-bank operands, as in a stand-alone launch,
// and allocates each phase's registers on its own -- inlined into the layer loop, the phases' state
// exceeded the register budget and spilled inside their inner loops.
__constant__ MkParams c_K;

constexpr int MK_SYNC_ABORT = 0;
constexpr int MK_SYNC_DONE = 1;
constexpr int MK_SYNC_PHASE = 2;

// The layer-specific fields of phase p (kind KIND of layer l), in the interface of HxPtrs.
template <int KIND>
struct MkPtrs {
  const MkParams& K;
  int l, p;
  unsigned dep_t;
  static constexpr int base() { return KIND == MK_QKV ? 0 : KIND == MK_O ? 3 : KIND == MK_GU ? 4 : 6; }
  __device__ __forceinline__ const gsdlq_hexmat_t& mat(int m) const {
    if constexpr (KIND == MK_HEAD) return K.lin[MK_HEAD].job.mat[m];
    else return K.layers[l].mats[base() + m];
  }
  __device__ __forceinline__ const float* norm_w() const {
    if constexpr (KIND == MK_QKV) return K.layers[l].attn_norm;
    else if constexpr (KIND == MK_GU) return K.layers[l].ffn_norm;
    else return K.lin[KIND].job.norm_w;
  }
  __device__ __forceinline__ int layer() const { return l; }
  __device__ __forceinline__ const CUtensorMap* tmap_codes(int m) const {
    return K.tmaps + 2 * (KIND == MK_HEAD ? 7 * K.n_layers + m : 7 * l + base() + m);
  }
  __device__ __forceinline__ const CUtensorMap* tmap_scales(int m) const { return tmap_codes(m) + 1; }
  __device__ __forceinline__ int input_mode() const {
    // the first layer's QKV reads the embedding row (the record holds the first layer's mode)
    if constexpr (KIND == MK_QKV) return l == 0 ? K.lin[MK_QKV].job.input_mode : GSDLQ_IN_RMSNORM;
    else return K.lin[KIND].job.input_mode;
  }
  __device__ __forceinline__ unsigned* ctl() const { return K.ctl + (size_t)CTL_WORDS * p; }
  // linear phases of a layer alternate workspaces QKV 0, O 1, gate/up 0, down 1 (head 0)
  __device__ __forceinline__ unsigned* cnt() const {
    return reinterpret_cast<unsigned*>(K.ws[(KIND == MK_O || KIND == MK_DN) ? 1 : 0]);
  }
  __device__ __forceinline__ unsigned long long* gacc() const {
    return reinterpret_cast<unsigned long long*>(K.ws[(KIND == MK_O || KIND == MK_DN) ? 1 : 0] + K.gacc_off[KIND]);
  }
  __device__ __forceinline__ const unsigned* dep() const { return p > 0 ? K.sync + MK_SYNC_PHASE + p - 1 : nullptr; }
  __device__ __forceinline__ unsigned dep_target() const { return dep_t; }
  __device__ __forceinline__ unsigned* done() const { return K.sync + MK_SYNC_PHASE + p; }
  __device__ __forceinline__ unsigned* abort() const { return K.sync + MK_SYNC_ABORT; }
  __device__ __forceinline__ unsigned trace_slot() const { return (unsigned)p; }
};

// completion count of a linear phase of kind KIND: its strips plus one per CTA (staging done)
template <int KIND>
__device__ __forceinline__ unsigned mk_lin_total(const MkParams& K) {
  return (unsigned)(K.lin[KIND].n_strips + (int)gridDim.x);
}

// MODE: 0 per-lane loads of any stream, 1 per-lane 16-byte loads (FULL streams), 2 the TMA ring
template <int KIND, int EPI, int MODE>
static __device__ __noinline__ void mk_linear(int l, int p, unsigned dep_t) {
  extern __shared__ __align__(1024) uint8_t smem[];
  hexmv_body<EPI, MODE >= 1, true, MODE == 2>(c_K.lin[KIND], MkPtrs<KIND>{c_K, l, p, dep_t}, smem);
}

template <int HD, int GQ>
static __device__ __noinline__ void mk_attention(int l, int p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const MkParams& K = c_K;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  uint8_t* scratch = smem + (HX_TAB_ABS - sbase) + 0x10000;
  const int tid = threadIdx.x;
  const int g = tid / AT_THREADS;  // two groups of AT_THREADS, named barriers 3 and 4
  AttnSmem<HD, GQ>* S = reinterpret_cast<AttnSmem<HD, GQ>*>(scratch) + g;
  const gsdlq_attn_job_t& J = K.attn;
  const int pos = *reinterpret_cast<const volatile int*>(J.pos_dev);
  const int len = (pos >= 0 && pos < J.max_seq) ? pos + 1 : 0;
  const int nsplit = K.nsplit;
  const int tps = max(1, (len + nsplit - 1) / nsplit);
  const int n_items = J.n_kv_heads * nsplit;
  const unsigned* dep = K.sync + MK_SYNC_PHASE + p - 1;
  const unsigned dep_t = mk_lin_total<MK_QKV>(K);
  unsigned* done = K.sync + MK_SYNC_PHASE + p;
  unsigned* abort = K.sync + MK_SYNC_ABORT;
  for (int it = blockIdx.x * 2 + g; it < n_items; it += gridDim.x * 2) {
    if (g == 0) {
      attn_body<HD, GQ, true, 3>(J, l, it / nsplit, it % nsplit, nsplit, tps, tid, *S, dep, dep_t, done, abort);
      attn_sync<3>();  // the group's buffers are reused by its next item
    } else {
      attn_body<HD, GQ, true, 4>(J, l, it / nsplit, it % nsplit, nsplit, tps, tid - AT_THREADS, *S, dep, dep_t, done,
                                 abort);
      attn_sync<4>();
    }
  }
}

template <int HD, int GQ, int MODE>
__global__ void __launch_bounds__(HX_THREADS, 1) decode_step_kernel() {
  extern __shared__ __align__(1024) uint8_t smem[];
  const MkParams& K = c_K;
  const int tid = threadIdx.x;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const uint32_t tab_off = HX_TAB_ABS - sbase;
  int* redi = reinterpret_cast<int*>(smem + tab_off - HX_RED_BYTES);
  __shared__ int s_last;
  if (tid == 0) redi[35] = -1;  // no decode table yet
  if (MODE == 2 && (tid & 31) == 0 && (tid >> 5) < HX_STREAM) {
    // each streaming warp's two TMA-ring barriers, and their parities, for the whole step
    const int warp = tid >> 5;
    const uint32_t bar0 = sbase + (tab_off - HX_RED_BYTES) + (uint32_t)(HX_MBAR_OFF + warp * 16);
    mbar_init(bar0, 1u);
    mbar_init(bar0 + 8u, 1u);
    mbar_fence_init();
    redi[HX_PH_OFF / 4 + warp] = 0;
  }
  __syncthreads();
  const int L = K.n_layers;
  for (int l = 0; l < L; ++l) {
    const int p = MK_PER_LAYER * l;
    mk_linear<MK_QKV, GSDLQ_EPI_ROPE_KV, MODE>(l, p, l > 0 ? mk_lin_total<MK_DN>(K) : 0u);
    __syncthreads();
    mk_attention<HD, GQ>(l, p + 1);
    __syncthreads();
    mk_linear<MK_O, GSDLQ_EPI_RESID, MODE>(l, p + 2, (unsigned)K.attn.n_kv_heads);
    __syncthreads();
    mk_linear<MK_GU, GSDLQ_EPI_SWIGLU, MODE>(l, p + 3, mk_lin_total<MK_O>(K));
    __syncthreads();
    mk_linear<MK_DN, GSDLQ_EPI_RESID, MODE>(l, p + 4, mk_lin_total<MK_GU>(K));
    __syncthreads();
  }
  if (K.with_head) {
    mk_linear<MK_HEAD, GSDLQ_EPI_STORE, MODE>(L - 1, MK_PER_LAYER * L, mk_lin_total<MK_DN>(K));
    __syncthreads();
  }
  // ---- end of the step: the last CTA advances the greedy state and zeroes the counters ------
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&K.sync[MK_SYNC_DONE], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0 && K.key != nullptr) {
    const unsigned long long k = *reinterpret_cast<volatile unsigned long long*>(K.key);
    const int t = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
    *K.token = t;
    if (K.out_ids != nullptr && *K.step < K.max_out) K.out_ids[*K.step] = t;
    *K.step += 1;
    *K.pos += 1;
    *K.key = 0ull;
  }
  for (int i = tid; i < K.ctl_words; i += HX_THREADS) K.ctl[i] = 0u;
  for (int i = MK_SYNC_PHASE + tid; i < MK_SYNC_PHASE + K.n_phases; i += HX_THREADS) K.sync[i] = 0u;
  if (tid == 0) K.sync[MK_SYNC_ABORT] = 0u;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    K.sync[MK_SYNC_DONE] = 0u;
  }
}

// ---- host side --------------------------------------------------------------------------------
int hexmv_plan(HexmvParams& P);
int hexmv_check_io(const HexmvParams& P);
bool hexmv_full(const HexmvParams& P);
bool hexmv_tma_ok(const HexmvParams& P);
int hexmv_encode_maps(const gsdlq_hexmat_t& M, CUtensorMap* codes, CUtensorMap* scales);

static_assert(sizeof(MkParams) <= 60 * 1024, "the decode kernel's parameters must fit the constant bank");

struct DecodePlan {
  int device = 0;
  int hd = 0, gq = 0, full = 0;
  int grid = 0, dyn_smem = 0;
  MkParams K;
  MkParams* K_pinned = nullptr;  // page-locked copy, the source of the per-step upload
  void* d_mem = nullptr;  // sync words, control blocks, strip workspaces, attention partials
};

using KernelFn = void (*)();

template <int HD, int GQ, int MODE>
static KernelFn mk_kernel_t() {
  if constexpr (attn_fits<HD, GQ>()) return decode_step_kernel<HD, GQ, MODE>;
  return nullptr;
}

// the (head_dim, query heads per kv head) shapes the decode kernel is built for, and their modes
static KernelFn mk_kernel(int hd, int gq, int mode) {
  if (hd == 128 && gq == 4) return mode == 2 ? mk_kernel_t<128, 4, 2>() : mode == 1 ? mk_kernel_t<128, 4, 1>() : mk_kernel_t<128, 4, 0>();
  if (hd == 128 && gq == 8) return mode == 1 ? mk_kernel_t<128, 8, 1>() : mode == 0 ? mk_kernel_t<128, 8, 0>() : nullptr;
  if (hd == 64 && gq == 4) return mode == 1 ? mk_kernel_t<64, 4, 1>() : mode == 0 ? mk_kernel_t<64, 4, 0>() : nullptr;
  if (hd == 32 && gq == 2) return mode == 0 ? mk_kernel_t<32, 2, 0>() : nullptr;
  return nullptr;
}

template <int HD, int GQ>
static size_t mk_attn_bytes_t() {
  return 2 * sizeof(AttnSmem<HD, GQ>);
}
static size_t mk_attn_bytes(int hd, int gq) {
  if (hd == 128 && gq == 4) return mk_attn_bytes_t<128, 4>();
  if (hd == 128 && gq == 8) return mk_attn_bytes_t<128, 8>();
  if (hd == 64 && gq == 4) return mk_attn_bytes_t<64, 4>();
  if (hd == 32 && gq == 2) return mk_attn_bytes_t<32, 2>();
  return 0;
}

static bool same_shape(const gsdlq_hexmat_t& a, const gsdlq_hexmat_t& b) {
  return a.rows == b.rows && a.cols == b.cols && a.k_dim == b.k_dim && a.radius == b.radius &&
         (a.unit_kink_off != nullptr) == (b.unit_kink_off != nullptr) && (a.unit_kinks != nullptr) == (b.unit_kinks != nullptr);
}

// Every layer must use the same shapes and the same activation buffers as the first: the kernel
// keeps one record per phase kind and only the matrices, the norm weight and the layer differ.
static bool same_job(const gsdlq_linear_job_t& a, const gsdlq_linear_job_t& b, bool input_may_differ) {
  if (a.n_mat != b.n_mat || a.epilogue != b.epilogue || a.x != b.x || a.eps != b.eps) return false;
  if (a.exchange || b.exchange) return false;  // (the persistent step has no tensor-parallel exchange)
  if (!input_may_differ && a.input_mode != b.input_mode) return false;
  for (int m = 0; m < a.n_mat; ++m) {
    if (!same_shape(a.mat[m], b.mat[m]) || a.y[m] != b.y[m]) return false;
  }
  return a.resid == b.resid && a.k_cache == b.k_cache && a.v_cache == b.v_cache && a.pos == b.pos &&
         a.rope_cs == b.rope_cs && a.max_seq == b.max_seq && a.head_dim == b.head_dim &&
         a.interleaved == b.interleaved && a.argmax_key == b.argmax_key;
}

}  // namespace gsdlq

using namespace gsdlq;

extern "C" int gsdlq_decode_plan_create(const gsdlq_decode_desc_t* d, gsdlq_decode_plan_t** out) {
  if (!d || !out || d->n_layers <= 0 || !d->layers) return GSDLQ_ERR_INVALID;
  *out = nullptr;
  const int L = d->n_layers;
  if (L > MK_MAX_LAYERS) return GSDLQ_ERR_UNSUPPORTED;
  const gsdlq_decode_layer_t& l0 = d->layers[0];
  const gsdlq_attn_job_t& A0 = l0.attn;
  if (A0.n_kv_heads <= 0 || A0.n_heads % A0.n_kv_heads) return GSDLQ_ERR_INVALID;
  const int hd = A0.head_dim, gq = A0.n_heads / A0.n_kv_heads;
  const int grid = num_sms();
  const bool with_head = d->head.n_mat != 0;
  DecodePlan* P = new DecodePlan();
  std::memset(&P->K, 0, sizeof(MkParams));
  MkParams& K = P->K;
  // ---- one shape record per kind, planned like a stand-alone launch of `grid` CTAs ------------
  const gsdlq_linear_job_t* tmpl[MK_KINDS] = {&l0.qkv, &l0.o, &l0.gate_up, &l0.down, &d->head};
  const int epi[MK_KINDS] = {GSDLQ_EPI_ROPE_KV, GSDLQ_EPI_RESID, GSDLQ_EPI_SWIGLU, GSDLQ_EPI_RESID, GSDLQ_EPI_STORE};
  int full = -1, st = GSDLQ_OK;
  size_t ws_need = 0;
  int ovf_max = 0, lacc_max = 0;
  for (int k = 0; k < MK_KINDS && st == GSDLQ_OK; ++k) {
    if (k == MK_HEAD && !with_head) break;
    HexmvParams& H = K.lin[k];
    H.job = *tmpl[k];
    // the decode kernel projects every linear's input itself (no forwarding between phases)
    H.job.fwd_acc = nullptr;
    H.job.lr_forwarded = 0;
    if (H.job.epilogue != epi[k]) st = GSDLQ_ERR_INVALID;
    if (st == GSDLQ_OK) st = hexmv_plan(H);
    if (st == GSDLQ_OK) st = hexmv_check_io(H);
    if (st != GSDLQ_OK) break;
    if (H.n_cta > grid) st = GSDLQ_ERR_UNSUPPORTED;
    // one stream mode serves every linear: 2 the TMA ring (opt-in), 1 16-byte loads (full units),
    // 0 any shape; the kernel takes the lowest mode any linear needs
    const int f = hexmv_full(H) ? (hexmv_tma_ok(H) ? 2 : 1) : 0;
    full = full < 0 ? f : std::min(full, f);
    ws_need = std::max(ws_need, hexmv_ws_bytes_for(H.n_strips, H.nmat));
    ovf_max = std::max(ovf_max, H.ovf_bytes);
    lacc_max = std::max(lacc_max, hx_lacc_bytes(H));
    K.gacc_off[k] = (int)((sizeof(unsigned) * (size_t)H.n_strips + 15) & ~size_t(15));
  }
  if (st == GSDLQ_OK && with_head && d->head.input_mode != GSDLQ_IN_RMSNORM) st = GSDLQ_ERR_UNSUPPORTED;
  if (st == GSDLQ_OK && (l0.o.input_mode != GSDLQ_IN_PLAIN || l0.down.input_mode != GSDLQ_IN_PLAIN ||
                         l0.gate_up.input_mode != GSDLQ_IN_RMSNORM))
    st = GSDLQ_ERR_UNSUPPORTED;
  // ---- per-layer records: matrices, norm weights; everything else must match the first layer --
  for (int l = 0; l < L && st == GSDLQ_OK; ++l) {
    const gsdlq_decode_layer_t& ly = d->layers[l];
    if (!same_job(ly.qkv, l0.qkv, true) || !same_job(ly.o, l0.o, false) || !same_job(ly.gate_up, l0.gate_up, false) ||
        !same_job(ly.down, l0.down, false))
      st = GSDLQ_ERR_UNSUPPORTED;
    if (l > 0 && ly.qkv.input_mode != GSDLQ_IN_RMSNORM) st = GSDLQ_ERR_UNSUPPORTED;
    if (ly.qkv.layer != l || ly.attn.layer != l) st = GSDLQ_ERR_UNSUPPORTED;
    const gsdlq_attn_job_t& a = ly.attn;
    if (a.q != A0.q || a.k_cache != A0.k_cache || a.v_cache != A0.v_cache || a.out != A0.out || a.pos_dev != A0.pos_dev ||
        a.n_heads != A0.n_heads || a.n_kv_heads != A0.n_kv_heads || a.head_dim != A0.head_dim ||
        a.max_seq != A0.max_seq || a.sm_scale != A0.sm_scale || a.block_table != nullptr)
      st = GSDLQ_ERR_UNSUPPORTED;
    // every matrix passes the stand-alone validation
    const gsdlq_linear_job_t* js[4] = {&ly.qkv, &ly.o, &ly.gate_up, &ly.down};
    for (int j = 0; j < 4 && st == GSDLQ_OK; ++j) {
      HexmvParams H{};
      H.job = *js[j];
      H.job.fwd_acc = nullptr;
      H.job.lr_forwarded = 0;
      st = hexmv_plan(H);
      if (st == GSDLQ_OK) st = hexmv_check_io(H);
    }
    MkLayer& R = K.layers[l];
    for (int m = 0; m < 3; ++m) R.mats[m] = ly.qkv.mat[m];
    R.mats[3] = ly.o.mat[0];
    R.mats[4] = ly.gate_up.mat[0];
    R.mats[5] = ly.gate_up.mat[1];
    R.mats[6] = ly.down.mat[0];
    R.attn_norm = ly.qkv.norm_w;
    R.ffn_norm = ly.gate_up.norm_w;
  }
  if (st == GSDLQ_OK && (!A0.q || !A0.k_cache || !A0.v_cache || !A0.out || !A0.pos_dev || A0.max_seq <= 0 ||
                         ((reinterpret_cast<uintptr_t>(A0.k_cache) | reinterpret_cast<uintptr_t>(A0.v_cache)) & 15u)))
    st = GSDLQ_ERR_INVALID;
  // not every attention shape has every stream mode built (the TMA ring only the most common
  // one): take the next lower mode that is
  while (st == GSDLQ_OK && full > 0 && mk_kernel(hd, gq, full) == nullptr) --full;
  const KernelFn fn = st == GSDLQ_OK ? mk_kernel(hd, gq, full) : nullptr;
  if (st == GSDLQ_OK && fn == nullptr) st = GSDLQ_ERR_UNSUPPORTED;
  if (st != GSDLQ_OK) {
    delete P;
    return st;
  }
  // ---- device memory: sync words | control blocks | 2 strip workspaces | attention scratch ----
  const int n_phases = MK_PER_LAYER * L + (with_head ? 1 : 0);
  const int nsplit = std::max(1, std::min(AT_MAX_SPLITS, 2 * grid / A0.n_kv_heads));
  const size_t sync_b = ((sizeof(unsigned) * (MK_SYNC_PHASE + n_phases)) + 255) & ~size_t(255);
  const size_t ctl_b = ((sizeof(unsigned) * (size_t)CTL_WORDS * n_phases) + 255) & ~size_t(255);
  const size_t ws_b = (ws_need + 255) & ~size_t(255);
  const size_t part_b = ((sizeof(float) * (size_t)A0.n_kv_heads * nsplit * gq * (hd + 2)) + 255) & ~size_t(255);
  const size_t aws_b = ((sizeof(unsigned) * (size_t)A0.n_kv_heads) + 255) & ~size_t(255);
  const size_t n_maps = 2 * (7 * (size_t)L + 1);
  const size_t maps_b = (sizeof(CUtensorMap) * n_maps + 255) & ~size_t(255);
  std::vector<CUtensorMap> maps(n_maps);
  if (full == 2) {
    for (int l = 0; l < L && st == GSDLQ_OK; ++l)
      for (int m = 0; m < 7 && st == GSDLQ_OK; ++m)
        st = hexmv_encode_maps(K.layers[l].mats[m], &maps[2 * (7 * l + m)], &maps[2 * (7 * l + m) + 1]);
    if (st == GSDLQ_OK && with_head)
      st = hexmv_encode_maps(d->head.mat[0], &maps[2 * 7 * L], &maps[2 * 7 * L + 1]);
    if (st != GSDLQ_OK) {
      delete P;
      return st;
    }
  }
  const size_t total = maps_b + sync_b + ctl_b + 2 * ws_b + part_b + aws_b;
  cudaError_t e = cudaGetDevice(&P->device);
  if (e == cudaSuccess) e = cudaMalloc(&P->d_mem, total);
  if (e == cudaSuccess) e = cudaMemset(P->d_mem, 0, total);
  if (e == cudaSuccess && full == 2)
    e = cudaMemcpy(P->d_mem, maps.data(), sizeof(CUtensorMap) * n_maps, cudaMemcpyHostToDevice);
  // dynamic shared memory: the table region, then max(activation overflow, attention groups) (the
  // host sizes for a zero reserved offset, as the stand-alone launch does)
  const size_t attn_b = mk_attn_bytes(hd, gq);
  // every linear phase's accumulator sits after the largest overflow region (and the ring)
  const size_t ring_b = full == 2 ? (size_t)ovf_max + HX_RING_BYTES : (size_t)ovf_max;
  for (int k = 0; k < MK_KINDS; ++k) K.lin[k].lacc_off = 0x10000 + (int)ring_b;
  P->dyn_smem = hx_dyn_smem(0) + (int)std::max<size_t>(ring_b + lacc_max, attn_b);
  if (e == cudaSuccess && P->dyn_smem > 227 * 1024) e = cudaErrorInvalidValue;
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, P->dyn_smem);
  int per_sm = 0;
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, HX_THREADS, P->dyn_smem);
  if (e == cudaSuccess && per_sm < 1) e = cudaErrorCooperativeLaunchTooLarge;
  if (e != cudaSuccess) {
    if (P->d_mem) cudaFree(P->d_mem);
    delete P;
    return e == cudaErrorInvalidValue ? GSDLQ_ERR_UNSUPPORTED : record_cuda_error(e);
  }
  K.tmaps = static_cast<const CUtensorMap*>(P->d_mem);
  uint8_t* base = static_cast<uint8_t*>(P->d_mem) + maps_b;
  K.sync = reinterpret_cast<unsigned*>(base);
  K.ctl = reinterpret_cast<unsigned*>(base + sync_b);
  K.ctl_words = CTL_WORDS * n_phases;
  K.n_phases = n_phases;
  K.ws[0] = base + sync_b + ctl_b;
  K.ws[1] = base + sync_b + ctl_b + ws_b;
  K.attn = A0;
  K.attn.fwd_acc = nullptr;
  K.attn.partial = reinterpret_cast<float*>(base + sync_b + ctl_b + 2 * ws_b);
  K.attn.workspace = reinterpret_cast<unsigned*>(base + sync_b + ctl_b + 2 * ws_b + part_b);
  K.n_layers = L;
  K.with_head = with_head ? 1 : 0;
  K.nsplit = nsplit;
  K.key = with_head ? d->argmax_key : nullptr;
  K.token = d->token;
  K.pos = d->pos;
  K.step = d->step;
  K.out_ids = d->out_ids;
  K.max_out = d->max_out;
  e = cudaMallocHost(reinterpret_cast<void**>(&P->K_pinned), sizeof(MkParams));
  if (e != cudaSuccess) {
    cudaFree(P->d_mem);
    delete P;
    return record_cuda_error(e);
  }
  std::memcpy(P->K_pinned, &K, sizeof(MkParams));
  P->hd = hd;
  P->gq = gq;
  P->full = full;
  P->grid = grid;
  *out = reinterpret_cast<gsdlq_decode_plan_t*>(P);
  return GSDLQ_OK;
}

extern "C" int gsdlq_decode_step(gsdlq_decode_plan_t* plan, gsdlq_stream_t stream) {
  if (!plan) return GSDLQ_ERR_INVALID;
  DecodePlan* P = reinterpret_cast<DecodePlan*>(plan);
  const KernelFn fn = mk_kernel(P->hd, P->gq, P->full);
  if (fn == nullptr) return GSDLQ_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P->grid);
  cfg.blockDim = dim3(HX_THREADS);
  cfg.dynamicSmemBytes = P->dyn_smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: phases wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // the plan's parameter block into the constant bank, ordered before the launch on its stream
  cudaError_t e = cudaMemcpyToSymbolAsync(c_K, P->K_pinned, sizeof(MkParams), 0, cudaMemcpyHostToDevice, cfg.stream);
  if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, fn);
  if (e != cudaSuccess) return record_cuda_error(e);
  return GSDLQ_OK;
}

extern "C" int gsdlq_decode_plan_destroy(gsdlq_decode_plan_t* plan) {
  if (!plan) return GSDLQ_OK;
  DecodePlan* P = reinterpret_cast<DecodePlan*>(plan);
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(P->device);
  cudaFree(P->d_mem);
  cudaFreeHost(P->K_pinned);
  cudaSetDevice(dev);
  delete P;
  return GSDLQ_OK;
}

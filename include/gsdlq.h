/*
 * gsdlq.h -- C ABI of libgsdlq_cuda.so, the B200 (sm_100a) decode engine for
 * GSD-LQ-packed decoders.
 *
 * Conventions
 *   - Every pointer argument that names tensor data is a DEVICE pointer unless
 *     stated otherwise.  The caller owns all buffers.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default
 *     stream).  All calls are asynchronous on that stream.
 *   - Every entry point returns an int status: GSDLQ_OK (0) or a negative
 *     GSDLQ_ERR_* code.  Argument errors are reported before any launch.
 *   - Kernels never trap.  A precondition that can only be checked on the
 *     device (a code >= n_pts, a kink column >= cols, pos >= max_seq, a table
 *     that is not an A2 lattice, a bounded wait that timed out) skips the
 *     offending access and sets a bit in a device flag word, read and cleared
 *     with gsdlq_device_flags().
 *
 * Section 1 lists drop-in replacements for the seven functions of the
 * reference C engine (gsd_lq_v2/gsd_lq_cpu_engine.c), bound by the reference
 * runtime through ctypes at gsd_lq_v2/gsd_lq_cpu_runtime.py:91-108.  They take
 * the same arguments in the same order with the same meaning, plus a trailing
 * stream, and return a status instead of void.  Section 2 lists the engine's
 * own fused entry points.
 */
#ifndef GSDLQ_H_
#define GSDLQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status and device flags ------------------------------------------------------- */
#define GSDLQ_OK 0
#define GSDLQ_ERR_INVALID (-1)     /* bad argument (shape, pointer, range) */
#define GSDLQ_ERR_CUDA (-2)        /* a CUDA runtime call failed; see gsdlq_last_cuda_error */
#define GSDLQ_ERR_UNSUPPORTED (-3) /* valid but not supported by this build */

#define GSDLQ_FLAG_BAD_CODE 0x1u   /* a code index >= n_pts was decoded as 0 */
#define GSDLQ_FLAG_BAD_KINK 0x2u   /* a kink column >= cols was skipped */
#define GSDLQ_FLAG_BAD_POS 0x4u    /* pos >= max_seq: KV store / attention skipped */
#define GSDLQ_FLAG_BAD_TABLE 0x8u  /* xy_table entry is not an A2 lattice point */
#define GSDLQ_FLAG_TIMEOUT 0x10u   /* a bounded device-side wait gave up */
#define GSDLQ_FLAG_BAD_TOKEN 0x20u /* token id >= vocab: embedding row skipped */
#define GSDLQ_FLAG_UNSUPPORTED 0x40u /* a kernel found a device limit it was not built for and did nothing */
#define GSDLQ_FLAG_RANGE 0x80u     /* a low-rank partial sum left the +-2^22 fixed-point range (clamped), or
                                      a scale above 5 reached the batched linear's fp16 weight parts */

typedef void *gsdlq_stream_t;

/* Human-readable name of a status code (static string). */
const char *gsdlq_status_string(int status);
/* The last cudaError_t seen by the library on this thread (0 if none). */
int gsdlq_last_cuda_error(void);
/* Copy the device flag word to *flags (host pointer), clear it, synchronise `stream`. */
int gsdlq_device_flags(unsigned int *flags, gsdlq_stream_t stream);
/* Library version string, e.g. "0.1.0 sm_100a". */
const char *gsdlq_version(void);

/* ---- 1. drop-in replacements for the reference C engine ------------------------------ */

/* out = x * (1/sqrt(mean(x^2) + eps)) * weight.
 * Replaces gsd_cpu_rmsnorm, gsd_lq_cpu_engine.c:67-82. */
int gsdlq_rmsnorm(const float *x, const float *weight, float *out, int dim, float eps,
                  gsdlq_stream_t stream);

/* y = a + b (y may alias a or b).  Replaces gsd_cpu_vec_add, gsd_lq_cpu_engine.c:85-94. */
int gsdlq_vec_add(float *y, const float *a, const float *b, int dim, gsdlq_stream_t stream);

/* out = silu(gate) * up (out may alias gate).  Replaces gsd_cpu_swiglu,
 * gsd_lq_cpu_engine.c:97-108. */
int gsdlq_swiglu(const float *gate, const float *up, float *out, int dim, gsdlq_stream_t stream);

/* tmp_k[j] = S[j] * sum_c x[c] * f16(Vt[j*cols + c]), j < k_dim <= 16.
 * Replaces gsd_cpu_lowrank_proj, gsd_lq_cpu_engine.c:111-127. */
int gsdlq_lowrank_proj(const float *x, const uint16_t *Vt, const float *S, float *tmp_k, int k_dim,
                       int cols, gsdlq_stream_t stream);

/* y[r] = sum_p (xy[c].x*x[2p] + xy[c].y*x[2p+1]) * f16(scales[(r*cols)/64 + p/32])
 *        + sum_{kinks of r} delta*x[col] + sum_j f16(U[r*k+j]) * tmp_k[j],
 * with c = codes[(r*cols)/2 + p].  cols % 64 == 0, k_dim <= 16, n_pts <= 256 and
 * xy_table an A2 lattice table (the reference's _get_turbo_codebook).
 * Replaces gsd_cpu_hex2d_matvec, gsd_lq_cpu_engine.c:130-183
 * (OpenCL twin: gsd_hex2d_matvec_fused, run_gpu_native_chat.py:196-267).
 * The library keeps one scratch area per device for this call (grown with cudaMalloc when a
 * larger matrix comes).  Back-to-back calls on one stream may share it; calls on DIFFERENT
 * streams of one device must not run at the same time (the reference's function is synchronous).
 * Callers with several streams use gsdlq_linear with a workspace per stream.
 * Width: the fused kernel holds a whole input row in shared memory (about 4 bytes per column), up to
 * GSDLQ_MATVEC_MAX_COLS columns.  Wider rows (to 65535, the reference's u16 kink column), and matrices
 * too tall for its per-CTA accumulator at such widths, go through the dequant-GEMM with one token
 * (gsdlq_hex2d_matmul's kernels, same result within the tolerance, codes 16-byte aligned), with a
 * second per-device scratch area.  gsdlq_linear and gsdlq_hex2d_matvec_noalloc return
 * GSDLQ_ERR_UNSUPPORTED for those shapes instead, before anything touches the device. */
#define GSDLQ_MATVEC_MAX_COLS 48640
int gsdlq_hex2d_matvec(const float *x, const uint8_t *codes, const uint16_t *scales,
                       const float *xy_table, const uint16_t *U, const float *tmp_k,
                       const uint32_t *kink_row_ptr, const uint16_t *kink_cols,
                       const float *kink_deltas, float *y, int rows, int cols, int k_dim,
                       int n_pts, gsdlq_stream_t stream);

/* RoPE on q (in place) and k; k (rotated) and v stored as fp16 at position pos of
 * a cache laid out [layer][max_seq_len][n_kv_heads][head_dim].  interleaved=1
 * rotates pairs (2i, 2i+1), 0 rotates (i, i + head_dim/2).  The rotation angles
 * are computed on the host with the reference's formula, so the result is
 * bit-identical to the reference given identical inputs.
 * Replaces gsd_cpu_rope_and_store_kv, gsd_lq_cpu_engine.c:186-262. */
int gsdlq_rope_and_store_kv(float *q, const float *k, const float *v, uint16_t *k_cache,
                            uint16_t *v_cache, int layer_idx, int pos, int n_heads, int n_kv_heads,
                            int head_dim, int max_seq_len, float rope_theta, int interleaved,
                            gsdlq_stream_t stream);

/* Decode attention for one query per head over positions 0..pos of the fp16
 * cache above; kv head = h / (n_heads / n_kv_heads).
 * Replaces gsd_cpu_gqa_attention, gsd_lq_cpu_engine.c:265-330. */
int gsdlq_gqa_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                        float *attn_out, int layer_idx, int pos, int n_heads, int n_kv_heads,
                        int head_dim, int max_seq_len, float sm_scale, gsdlq_stream_t stream);

/* ---- 2. engine entry points ----------------------------------------------------------- */

/* HOST function.  A2 lattice table of `radius` into xy_out (2*max_pts floats,
 * host memory), bit-identical to _get_turbo_codebook (gsd_lq_cpu_runtime.py:111-118).
 * Returns n_pts (127 for radius 6, 217 for radius 8), or GSDLQ_ERR_INVALID. */
int gsdlq_codebook(int radius, float *xy_out, int max_pts);

/* W[r,c] = xy[code][c&1] * f16->f32(scale): the dequantised weight as the
 * reference's NumPy path defines it (gsd_lq_cpu_runtime.py:281-284), bit-exact. */
int gsdlq_dequant(const uint8_t *codes, const uint16_t *scales, const float *xy_table, float *w,
                  int rows, int cols, int n_pts, gsdlq_stream_t stream);

/* Greedy pick over n logits with the reference's nan_to_num + first-maximum rule
 * (gsd_lq_cpu_runtime.py:422-425).  *out_index (device int) receives the index. */
int gsdlq_argmax(const float *logits, int n, int *out_index, gsdlq_stream_t stream);

/* Packer: lattice codes, fp16 group scales and the fp32 residual W - dequant of a
 * row-major fp32 [rows, cols] matrix.  Bit-identical to the NumPy packer
 * (gsdlq_b200.packer.quantize_lattice).  No reference counterpart: the
 * reference ships no packer. */
int gsdlq_pack_lattice(const float *w, int rows, int cols, int radius, uint8_t *codes,
                       uint16_t *scales, float *residual, gsdlq_stream_t stream);

/* One packed linear (reference layout, device pointers). */
typedef struct gsdlq_hexmat {
  const uint8_t *codes;       /* [rows*cols/2]                          */
  const uint16_t *scales;     /* [rows*cols/64] fp16                    */
  const uint16_t *U;          /* [rows*k_dim] fp16 (unused if k_dim==0) */
  const float *S;             /* [k_dim]                                */
  const uint16_t *Vt;         /* [k_dim*cols] fp16                      */
  const uint32_t *row_ptr;    /* [rows+1] CSR kink offsets              */
  const uint16_t *kink_cols;  /* [nnz]                                  */
  const float *kink_deltas;   /* [nnz]                                  */
  int rows, cols, k_dim, radius;
  /* Optional (gsdlq_linear only; NULL = use the CSR arrays above): the same kinks regrouped
   * per work unit of 16 rows x 512 columns, built by gsdlq_unit_kinks.  unit_kink_off has
   * ceil(rows/16) * ceil(cols/512) + 1 offsets; entry i of unit_kinks is two words
   * (col | row_in_strip << 16, fp32 delta bits), rows then columns ascending within a unit. */
  const uint32_t *unit_kink_off;
  const uint32_t *unit_kinks;
} gsdlq_hexmat_t;

#define GSDLQ_EPI_STORE 0   /* y[m][r] = W_m x                                            */
#define GSDLQ_EPI_RESID 1   /* y[0][r] = resid[r] + W_0 x   (y may alias resid)              */
#define GSDLQ_EPI_SWIGLU 2  /* y[0][r] = silu(W_0 x) * (W_1 x)   (pair of equal-shape mats)  */
#define GSDLQ_EPI_ROPE_KV 3 /* mats = Q, K, V: y[0] = RoPE(Qx); RoPE(Kx), Vx -> fp16 KV cache */

#define GSDLQ_IN_PLAIN 0    /* input = x                                                  */
#define GSDLQ_IN_RMSNORM 1  /* input = rmsnorm(x) * norm_w                                */
#define GSDLQ_IN_EMBED 2    /* input = rmsnorm(f32(embed[*token])) * norm_w; CTA 0 writes the
                               raw row to x_out (the residual stream)                      */

/* A tensor-parallel exchange among the ranks of one node (gsdlq_comm_create; see that section). */
#define GSDLQ_IPC_HANDLE_BYTES 64
typedef struct gsdlq_comm gsdlq_comm_t;  /* opaque */

/* L2 prefetch list of a launch (engine use; no counterpart in the reference): byte ranges of
 * device memory that a LATER launch will read -- the next linears' packed weights -- fetched into
 * the L2 cache while this launch runs, so that HBM keeps streaming across the gaps between
 * dependent launches.  Each range must start 16-byte aligned and span a multiple of 16 bytes; the
 * ranges are split evenly over the launch's CTAs and issued as bulk L2 prefetches at their start.
 * n = 0: none.  Prefetches change no result. */
#define GSDLQ_MAX_PREFETCH 16
typedef struct gsdlq_prefetch {
  const void *ptr[GSDLQ_MAX_PREFETCH];
  uint64_t bytes[GSDLQ_MAX_PREFETCH];
  int n;
} gsdlq_prefetch_t;

/* A fused packed-linear launch: up to three matrices that share one input,
 * the low-rank projection computed inside the same kernel, and an epilogue. */
typedef struct gsdlq_linear_job {
  gsdlq_hexmat_t mat[3];
  int n_mat;
  int input_mode;             /* GSDLQ_IN_*                                   */
  const float *x;             /* [cols] (PLAIN, RMSNORM)                      */
  const float *norm_w;        /* [cols] (RMSNORM, EMBED)                      */
  float eps;
  const uint16_t *embed;      /* [vocab, cols] fp16 (EMBED)                   */
  const int *token;           /* device token id (EMBED)                      */
  int vocab;
  float *x_out;               /* EMBED: receives the f32 embedding row        */
  int epilogue;               /* GSDLQ_EPI_*                                  */
  float *y[3];
  const float *resid;         /* RESID                                        */
  /* ROPE_KV */
  uint16_t *k_cache, *v_cache; /* [layers][max_seq][n_kv][head_dim] fp16       */
  const int *pos;             /* device position                              */
  const float *rope_cs;       /* [max_seq][head_dim/2] (cos, sin) pairs        */
  int layer, max_seq, head_dim, interleaved;
  /* optional fused greedy argmax of y[0] (EPI_STORE): atomicMax of a 64-bit
   * (value, ~index) key; the key must start at 0 */
  unsigned long long *argmax_key;
  int argmax_index_base;      /* added to the row index in the key (vocab-parallel LM head) */
  /* Low-rank forwarding (optional; engine use).  A launch whose output is the NEXT linear's input
   * adds that linear's projection of it, strip by strip, to the next launch's accumulators:
   * fwd_acc[lr_off(m) + j] += round(2^32 * sum_r Vt_m[j][r] * w[r] * out[r]) (two's-complement
   * 64-bit), over the rows r it finished, for the next linear's matrices m (fwd_vt[m], fwd_k[m]
   * rows of [cols] fp16) and w = fwd_norm_w (1 when NULL).  out is the epilogue's output (the new
   * residual for RESID, the SwiGLU product for SWIGLU, y for STORE).  fwd_acc is the next launch's
   * workspace + 64 bytes (its accumulator words), so the next launch's workspace must be zero at
   * this launch's start.  The next launch sets lr_forwarded = 1: it skips its own projection and
   * scales the accumulators by its 1/rms (RMSNORM input) and S. */
  const uint16_t *fwd_vt[3];
  int fwd_k[3];
  const float *fwd_norm_w;
  unsigned long long *fwd_acc;
  int lr_forwarded;
  gsdlq_prefetch_t prefetch;  /* optional L2 prefetch of later launches' weights */
  /* Tensor parallelism (optional; RESID epilogue of one matrix): a connected exchange (host
   * handle).  Every rank then finishes each strip as
   *   y[r] = ((resid[r] + p_0[r]) + p_1[r]) + ... + p_{W-1}[r],
   * p_w = rank w's partial W x, exchanged through the peers' buffers strip by strip -- the
   * all-reduce of the row-parallel O and down projections fused into their epilogue, the same bits
   * on every rank; low-rank forwarding (fwd_acc) is applied to the summed y.  Every rank must
   * launch the same sequence of such jobs. */
  gsdlq_comm_t *exchange;
} gsdlq_linear_job_t;

/* Bytes of device workspace a gsdlq_linear launch of `job` needs (host pointers). */
int gsdlq_linear_ws_size(const gsdlq_linear_job_t *job, size_t *bytes);

/* Launch a fused packed linear.  `job` is a HOST pointer (read during the call).
 * `workspace`: device memory of at least gsdlq_linear_ws_size bytes, 16-byte
 * aligned, all zero before its first use.  Every launch leaves the bytes it used
 * at zero again, so one workspace serves any number of launches, of any shape,
 * that do not overlap in time.  Two launches that may overlap -- consecutive
 * launches on one stream, which use programmatic dependent launch -- need
 * distinct workspaces. */
int gsdlq_linear(const gsdlq_linear_job_t *job, void *workspace, size_t workspace_bytes,
                 gsdlq_stream_t stream);

/* Regroup a packed linear's CSR kinks into the per-unit lists of gsdlq_hexmat_t (device
 * pointers).  unit_kink_off: ceil(rows/16) * ceil(cols/512) + 1 words; unit_kinks: 2 * nnz words.
 * Engine layout with no reference counterpart: the fused linear then applies the kinks of each
 * 16 x 512 work unit in the streaming loop instead of in separate per-row passes. */
int gsdlq_unit_kinks(const uint32_t *row_ptr, const uint16_t *kink_cols, const float *kink_deltas,
                     int rows, int cols, uint32_t *unit_kink_off, uint32_t *unit_kinks,
                     gsdlq_stream_t stream);

/* Size of the library's fixed device scratch array used by gsdlq_hex2d_matvec_noalloc, and the
 * most 16-row strips a call may have: a launch needs 768 + 132 * strips bytes of it (control
 * words, one count and sixteen 8-byte partial sums per strip), so at most
 * (GSDLQ_NOALLOC_WS_BYTES - 768) / 132 = 31 769 strips, i.e. rows <= 508 304. */
#define GSDLQ_NOALLOC_WS_BYTES (4u << 20)
#define GSDLQ_NOALLOC_MAX_STRIPS 31769u

/* gsdlq_hex2d_matvec without any device allocation.  No counterpart in the reference:
 * the reference's matvec runs on the host and needs no scratch.
 *
 * Who it is for: gsdlq_hex2d_matvec keeps the reference signature, which has no
 * workspace argument, so on first use it allocates its scratch with cudaMalloc.
 * Some callers cannot allow that: a host that has handed all device memory to its own
 * allocator or to a fixed budget, and latency-critical loops where cudaMalloc/cudaFree
 * may synchronise the device.  This variant takes the same arguments and gives the same
 * result.  Its scratch is a file-scope device array of GSDLQ_NOALLOC_WS_BYTES (4 MiB) that
 * every GPU loading this library holds until the process exits.
 *
 * - The first call on a device looks up the array's device address (cudaGetSymbolAddress,
 *   with that device current) and keeps it.  Make that first call before any stream
 *   capture begins.
 * - Each call clears the scratch bytes it needs with cudaMemsetAsync on `stream`, then
 *   launches.  It calls no cudaMalloc, cudaFree or other allocating routine.
 * - All calls share the one array.  Calls that may overlap on the GPU (different streams,
 *   or different host threads without ordering) race on it and give wrong results.
 * - Argument errors and a matrix of more than GSDLQ_NOALLOC_MAX_STRIPS strips of 16 rows
 *   (rows > 508 304) return GSDLQ_ERR_INVALID or GSDLQ_ERR_UNSUPPORTED before anything
 *   touches the device.  (The planner of every packed-linear entry point has a lower limit
 *   of its own, 127 strips per SM -- 18 796 strips, 300 736 rows, on a 148-SM B200 -- and
 *   returns GSDLQ_ERR_UNSUPPORTED above it, so the scratch is never the binding limit there.) */
int gsdlq_hex2d_matvec_noalloc(const float *x, const uint8_t *codes, const uint16_t *scales,
                               const float *xy_table, const uint16_t *U, const float *tmp_k,
                               const uint32_t *kink_row_ptr, const uint16_t *kink_cols,
                               const float *kink_deltas, float *y, int rows, int cols, int k_dim,
                               int n_pts, gsdlq_stream_t stream);

/* Split-KV decode attention.  q is already rotated.  pos is read from *pos_dev
 * when non-NULL (CUDA-graph friendly), else pos_val.  The cache layout is the
 * reference's [layer][max_seq][n_kv][head_dim] fp16 when block_table is NULL,
 * else a paged pool [page][page_size][n_kv][head_dim] with block_table[t/page_size]
 * giving the page of position t.  partial/workspace: see gsdlq_attention_ws_size. */
typedef struct gsdlq_attn_job {
  const float *q;
  const uint16_t *k_cache, *v_cache;
  float *out;
  const int *pos_dev;
  int pos_val;
  int layer, n_heads, n_kv_heads, head_dim, max_seq;
  float sm_scale;
  const int *block_table;
  int page_size;
  float *partial;
  unsigned int *workspace;
  /* low-rank forwarding into the next linear (the O projection; see gsdlq_linear_job_t): each
   * combined kv head adds fwd_vt[j][c] * out[c] over its head columns c to fwd_acc[j], j < fwd_k */
  const uint16_t *fwd_vt;
  int fwd_k;
  unsigned long long *fwd_acc;
  gsdlq_prefetch_t prefetch;  /* optional L2 prefetch of later launches' weights */
} gsdlq_attn_job_t;

/* Bytes of `partial` (floats) and `workspace` (uints) a gsdlq_attention call needs. */
int gsdlq_attention_ws_size(int n_heads, int n_kv_heads, int head_dim, int max_seq,
                            size_t *partial_bytes, size_t *workspace_bytes);
int gsdlq_attention(const gsdlq_attn_job_t *job, gsdlq_stream_t stream);

/* Device-side greedy bookkeeping after a step whose LM head fed *argmax_key:
 * *token = argmax index, out_ids[*step] = token (when out_ids != NULL and
 * *step < max_out), *step += 1, *pos += 1, *argmax_key = 0.  One thread; lets a
 * captured decode step be replayed back to back without host round trips. */
int gsdlq_greedy_advance(unsigned long long *argmax_key, int *token, int *pos, int *step, int *out_ids,
                         int max_out, gsdlq_stream_t stream);

/* gsdlq_greedy_advance with an EOS stop (the reference chat loop, run_gpu_native_chat.py:1142-1144):
 * when the picked token equals eos_id, *done is set to 1 and token, pos, step and out_ids stay as
 * they are (the EOS token is not stored); while *done is set, calls only clear *argmax_key.
 * eos_id < 0: no stop. */
int gsdlq_advance_eos(unsigned long long *argmax_key, int *token, int *pos, int *step, int *out_ids, int max_out,
                      int eos_id, int *done, gsdlq_stream_t stream);

/* ---- Temperature + top-p sampling (gsd_lq_cpu_runtime.py:422-443, sample_token) ------------------
 * One pick from logits[n] (device) with the reference's rules: NaN -> -1e4, +-inf -> 100 / -1e4;
 * greedy argmax when temperature <= 0; p = softmax(logits / max(temperature, 1e-4)); the nucleus is
 * the descending-order prefix up to and including the first entry whose running sum exceeds top_p
 * (the top entry alone when none does); the pick is the first nucleus entry whose running share of
 * the nucleus exceeds the uniform draw u in [0, 1) -- the draw np.random.choice makes
 * (np.random.random_sample()), so that picks match the reference's under the same NumPy seed.
 * u: device double; u_index: NULL (u[0]) or a device int selecting u[*u_index] (the decode step, for a
 * captured loop).  Writes *out_index and / or *argmax_key (in the greedy-argmax key format, so that
 * gsdlq_greedy_advance / gsdlq_advance_eos take the pick).  work: n floats of device scratch.
 * Running sums are exact here (2^-56 fixed point) and rounded in the reference: picks agree except
 * where a target lies within rounding distance of a running sum (top_p >= 1 is one such case), and
 * equal probabilities are taken in ascending index order (NumPy's argsort order for them is
 * unspecified). */
int gsdlq_sample_work_size(int n, size_t *bytes);
int gsdlq_sample_top_p(const float *logits, int n, float temperature, float top_p, const double *u,
                       const int *u_index, void *work, size_t work_bytes, unsigned long long *argmax_key,
                       int *out_index, gsdlq_stream_t stream);

/* HOST function: (cos, sin) of the RoPE angles for positions [0, max_seq) into
 * table (host, max_seq*head_dim floats), computed with the reference's formula
 * (gsd_lq_cpu_engine.c:215-218) so that rotations match it bit for bit. */
int gsdlq_rope_table(float *table, int max_seq, int head_dim, float rope_theta);

/* ---- Batched packed linear (B tokens) ---------------------------------------------------------
 * y[b] = gsd_cpu_hex2d_matvec(gsd_cpu_lowrank_proj(x[b])) for b < batch (gsd_lq_cpu_engine.c:111-183
 * applied to each token), as one dequant-GEMM on the tcgen05 tensor cores (accumulators in tensor
 * memory): the codes are decoded once per launch for all tokens; the kink and low-rank terms are
 * added in fp32 by a separate sparse pass.  x: [batch][cols] fp32, 16-byte aligned; y: [batch][rows]
 * fp32 (written here); work: device scratch of at least gsdlq_hex2d_matmul_work_size(batch, cols)
 * bytes, 1024-byte aligned (per-token maxima and low-rank projections, and the activations converted
 * once into the tensor cores' operand layout and transposed).  1 <= batch <= GSDLQ_MATMUL_MAX_BATCH,
 * cols a multiple of 64 and at most 65535, k_dim <= 16, n_pts <= 256, codes and Vt 16-byte aligned,
 * xy_table the A2 lattice points (as the matvec requires); above 32 tokens scales at most 5
 * (GSDLQ_FLAG_RANGE otherwise).  Weights and activations enter the tensor cores as fp16 hi + lo parts (about 22
 * significant bits): results match the per-token matvec to about 1e-6 relative.  The partial sums
 * are added with atomics, so the last bits may differ between runs. */
#define GSDLQ_MATMUL_MAX_BATCH 128
int gsdlq_hex2d_matmul_work_size(int batch, int cols, size_t *bytes);
int gsdlq_hex2d_matmul(const float *x, int batch, const uint8_t *codes, const uint16_t *scales,
                       const float *xy_table, const uint16_t *U, const float *S, const uint16_t *Vt,
                       const uint32_t *kink_row_ptr, const uint16_t *kink_cols, const float *kink_deltas,
                       float *y, void *work, size_t work_bytes, int rows, int cols, int k_dim, int n_pts,
                       gsdlq_stream_t stream);

/* ---- Chunked prefill: the per-token operations over the n rows of a chunk ---------------------
 * No counterpart in the reference, whose prefill runs forward_token once per prompt token
 * (run_gpu_native_chat.py:1128-1131): each of these applies the reference's per-token operation to
 * every row of a chunk of n tokens at positions pos0 .. pos0 + n - 1 ([n][dim] fp32 rows, device).
 *   embed_rows:     out[t] = f32(embed[ids[t]]) (ids: device int32)
 *   rmsnorm_rows:   gsd_cpu_rmsnorm of every row (gsd_lq_cpu_engine.c:67-82)
 *   rope_kv_rows:   gsd_cpu_rope_and_store_kv of every row, interleaved pairs, angles from the
 *                   gsdlq_rope_table table rope_cs [max_seq][head_dim/2] (gsd_lq_cpu_engine.c:186-262)
 *   attention_rows: gsd_cpu_gqa_attention of row t at position pos0 + t: causal over the cache
 *                   (gsd_lq_cpu_engine.c:265-330); head_dim 64 or 128, n_heads / n_kv_heads <= 8;
 *                   q, out, work 16-byte aligned; work (device) of at least the bytes
 *                   gsdlq_attention_rows_work_size gives for (n, n_heads, head_dim) */
int gsdlq_embed_rows(const uint16_t *embed, const int *ids, int n, int vocab, int dim, float *out,
                     gsdlq_stream_t stream);
int gsdlq_rmsnorm_rows(const float *x, const float *w, float *out, int n, int dim, float eps, gsdlq_stream_t stream);
int gsdlq_rope_kv_rows(float *q, const float *k, const float *v, uint16_t *k_cache, uint16_t *v_cache,
                       const float *rope_cs, int layer, int pos0, int n, int n_heads, int n_kv_heads, int head_dim,
                       int max_seq, gsdlq_stream_t stream);
int gsdlq_attention_rows_work_size(int n, int n_heads, int head_dim, size_t *bytes);
int gsdlq_attention_rows(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, float *out, void *work,
                         size_t work_bytes, int layer, int pos0, int n, int n_heads, int n_kv_heads, int head_dim,
                         int max_seq, float sm_scale, gsdlq_stream_t stream);

/* ---- Batched decode: B independent sequences, one token each per step -------------------------
 * No counterpart in the reference (batch 1 only).  Each sequence has its own KV cache, seq_stride
 * elements after the previous one's ([B][layers][max_seq][n_kv_heads][head_dim] fp16 for
 * seq_stride = layers * max_seq * n_kv_heads * head_dim), and its own position pos[b] (device ints).
 *   rope_kv_batch:         gsd_cpu_rope_and_store_kv (gsd_lq_cpu_engine.c:186-262) of row b at pos[b]
 *                          into sequence b's cache (interleaved pairs, angles from rope_cs)
 *   attention_decode_batch: gsd_cpu_gqa_attention (gsd_lq_cpu_engine.c:265-330) of row b over
 *                          positions 0 .. pos[b] of sequence b's cache; head_dim 64 or 128, 1, 2, 4,
 *                          6 or 8 query heads per kv head; work: gsdlq_attention_rows_work_size(B, ...)
 *                          row_stride / q_stride: elements between consecutive rows of q (and k, v),
 *                          0 for packed rows -- a nonzero stride reads q, k, v out of one linear's output
 *                          over the stacked q, k and v rows
 *   swiglu_rows:           gsd_cpu_swiglu (gsd_lq_cpu_engine.c:97-108) of rows laid out [gate | up]
 *   argmax_rows:           greedy pick of every row of logits[rows][n] (the reference's greedy rule)
 *                          into ids[b]; with pos: out_ids[b * out_stride + pos[b] + 1] = pick (when
 *                          out_ids and inside out_stride) and pos[b] += 1 */
int gsdlq_rope_kv_batch(float *q, const float *k, const float *v, int row_stride, uint16_t *k_cache,
                        uint16_t *v_cache, size_t seq_stride, const float *rope_cs, int layer, const int *pos, int batch,
                        int n_heads, int n_kv_heads, int head_dim, int max_seq, gsdlq_stream_t stream);
int gsdlq_attention_decode_batch(const float *q, int q_stride, const uint16_t *k_cache, const uint16_t *v_cache,
                                 size_t seq_stride, float *out, void *work, size_t work_bytes, int layer, const int *pos,
                                 int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq, float sm_scale,
                                 gsdlq_stream_t stream);
int gsdlq_swiglu_rows(const float *gate_up, float *out, int rows, int n, gsdlq_stream_t stream);
int gsdlq_argmax_rows(const float *logits, int rows, int n, int *ids, int *pos, int *out_ids, int out_stride,
                      gsdlq_stream_t stream);

/* ---- The whole decode step in one launch ----------------------------------------------------
 * Engine-level entry point with no single reference counterpart: the reference's
 * Model.forward_token (run_gpu_native_chat.py:921-984) walks the layers on the host, one kernel
 * per operation; this runs the same sequence -- per layer QKV (+RoPE, KV append), attention, O
 * (+residual), gate/up (+SwiGLU), down (+residual), then the LM head with the greedy argmax and
 * the greedy bookkeeping of gsdlq_greedy_advance -- as one cooperative launch of one CTA per SM
 * whose phases wait on one another through device counters.
 *
 * The jobs are the ones gsdlq_linear / gsdlq_attention take (their workspace fields are ignored:
 * the plan owns its scratch).  Requirements: every linear has the same stream shape (all with
 * cols a multiple of 512 and 16-byte aligned scales, or none), the attention shape (head_dim,
 * n_heads / n_kv_heads) is one the library is built for (128/4, 128/8, 64/4, 32/2), contiguous
 * KV cache (no block table); otherwise gsdlq_decode_plan_create returns GSDLQ_ERR_UNSUPPORTED and
 * the caller runs the per-operation launches.  Results equal the per-operation launches' to float
 * rounding (the attention splits the sequence differently).  Each step first copies the plan's
 * parameter block into the library's constant memory on `stream`, so the steps of all plans of
 * one device must not overlap on the GPU (use one stream, or ordered streams). */
/* ---- Tensor-parallel exchange (engine use) -----------------------------------------------------
 * No counterpart in the reference, which runs on one device.  A one-shot all-reduce among the W
 * ranks (one process per GPU) of one node, through each rank's exchange buffer mapped into every
 * peer with CUDA IPC: every rank stores its values into every peer's receive slots over NVLink,
 * raises a flag there, waits (bounded: 1 s, then GSDLQ_FLAG_TIMEOUT) for every peer's flag and sums
 * the slots in rank order, so all ranks hold the same bits.  Every rank must make the same calls in
 * the same order.  No TMA and no multicast are used.
 *   create:  allocates this rank's buffer (for vectors of up to n_max floats) and writes its
 *            GSDLQ_IPC_HANDLE_BYTES-byte IPC handle to ipc_handle;
 *   connect: handles = the W ranks' handles, rank-major; opens the peers' buffers;
 *   allreduce_sum: x[n] (16-byte aligned, device) := the sum over ranks, in place;
 *   allreduce_max_u64: *key := the maximum over ranks (the vocab-parallel greedy argmax key).
 * Both are stream-ordered kernels (capturable into a CUDA graph) that read their input after the
 * previous kernel on the stream has completed. */
int gsdlq_comm_create(int world, int rank, int n_max, gsdlq_comm_t **comm, void *ipc_handle);
int gsdlq_comm_connect(gsdlq_comm_t *comm, const void *handles);
int gsdlq_comm_allreduce_sum(gsdlq_comm_t *comm, float *x, int n, gsdlq_stream_t stream);
int gsdlq_comm_allreduce_max_u64(gsdlq_comm_t *comm, unsigned long long *key, gsdlq_stream_t stream);
int gsdlq_comm_destroy(gsdlq_comm_t *comm);

typedef struct gsdlq_decode_layer {
  gsdlq_linear_job_t qkv;      /* epilogue GSDLQ_EPI_ROPE_KV */
  gsdlq_attn_job_t attn;
  gsdlq_linear_job_t o;        /* GSDLQ_EPI_RESID */
  gsdlq_linear_job_t gate_up;  /* GSDLQ_EPI_SWIGLU */
  gsdlq_linear_job_t down;     /* GSDLQ_EPI_RESID */
} gsdlq_decode_layer_t;

typedef struct gsdlq_decode_desc {
  int n_layers;
  const gsdlq_decode_layer_t *layers;  /* host array of n_layers */
  gsdlq_linear_job_t head;             /* GSDLQ_EPI_STORE with argmax_key; n_mat 0: no head
                                          (a prefill step: layers only, no greedy bookkeeping) */
  /* greedy bookkeeping after the head (as gsdlq_greedy_advance); argmax_key NULL: none */
  unsigned long long *argmax_key;
  int *token, *pos, *step, *out_ids;
  int max_out;
} gsdlq_decode_desc_t;

typedef struct gsdlq_decode_plan gsdlq_decode_plan_t;  /* opaque */

/* Plan the step (validates every job, allocates the plan's device scratch). */
int gsdlq_decode_plan_create(const gsdlq_decode_desc_t *desc, gsdlq_decode_plan_t **plan);
/* One decode token: a single launch on `stream`. */
int gsdlq_decode_step(gsdlq_decode_plan_t *plan, gsdlq_stream_t stream);
int gsdlq_decode_plan_destroy(gsdlq_decode_plan_t *plan);

#ifdef __cplusplus
}
#endif
#endif /* GSDLQ_H_ */

/*
 * flashborn_b200.h -- C ABI of the B200 (sm_100a) flash-Born attention library.
 *
 * Born attention (softmax-free; no exp, no running max):
 *
 *   plain     a_ij = max(0, scale_h * <q_i, k_j>) * valid(i, j)       p_ij = a_ij^2
 *   purified  u_ij = max(0, gamma_h * (<q_i, k_j> - tau_h)) * valid,  b_ij = max(0, <q_i, k_j>) * valid
 *             p_ij = u_ij^4 + eps_base * b_ij^2
 *   both      Z_i = sum_j p_ij + eps          O_i = (sum_j p_ij v_j) / Z_i
 *
 *   valid(i, j) = (j <= i if causal) & (i - j < window if window > 0) & (doc_i == doc_j if doc ids)
 *
 * Every entry point replaces one host->device launch site of the reference
 * (qdlblocks, src/qdlblocks/kernels/flash_born.py) and keeps its argument meaning:
 *
 *   fb_born_fwd            _flash_born_fwd_kernel[grid](...)                    flash_born.py:475-513
 *   fb_born_bwd            _flash_born_bwd_kernel + _flash_born_bwd_dq_kernel   flash_born.py:554-612
 *   fb_purified_born_fwd   _flash_purified_born_fwd_kernel[grid](...)          flash_born.py:1110-1147
 *   fb_purified_born_bwd   _flash_purified_born_bwd(_dq)_kernel                 flash_born.py:1197-1262
 *
 * Conventions
 *   - The caller owns every buffer (out, z, dq, dk, dv, dscale, dtau, workspace); the library
 *     never allocates or frees device memory.  One exception: fb_born_bwd_static_scratch's
 *     fixed FB_STATIC_SCRATCH_BYTES array, part of the library's device module (see there).
 *   - Tensors are (B, H, T, D) with arbitrary element strides (the innermost stride must be 1 for
 *     the tensor-core path; other layouts run on the general path). doc_ids is (B, T) int32.
 *   - scale / tau are device fp32 vectors of 1 (shared) or H (per head) elements.
 *   - dscale / dtau are device fp32 vectors of scale_numel / tau_numel elements; the backward
 *     ACCUMULATES into them (zero them first, as the reference does at flash_born.py:536).
 *   - z is (B, H, T) contiguous fp32 and holds sum_j p_ij + eps (saved for the backward).
 *   - All work is enqueued on `stream` (a cudaStream_t, NULL = legacy default stream);
 *     nothing synchronises the host.
 *   - Errors are returned as FB_* status codes (never a device trap). Errors found on the device
 *     (an mbarrier wait that ran past its bound) are latched in a device status word read by
 *     fb_device_status().
 */
#ifndef FLASHBORN_B200_H_
#define FLASHBORN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FB_ABI_VERSION 4

#if defined(__GNUC__)
#define FB_API __attribute__((visibility("default")))
#else
#define FB_API
#endif

/* Status codes. */
enum {
  FB_OK = 0,
  FB_ERR_SHAPE = 1,       /* B/H/T/D out of range, mismatched shapes */
  FB_ERR_DTYPE = 2,       /* unsupported element type combination */
  FB_ERR_ALIGN = 3,       /* pointer or stride alignment */
  FB_ERR_ARG = 4,         /* null pointer, bad scale/tau length, bad window */
  FB_ERR_LAUNCH = 5,      /* CUDA launch or attribute error (see fb_last_cuda_error) */
  FB_ERR_TIMEOUT = 6,     /* a bounded device-side wait gave up (device status word) */
  FB_ERR_WORKSPACE = 7,   /* workspace missing or too small */
  FB_ERR_NO_DEVICE = 8,   /* no CUDA device / driver entry point unavailable */
  FB_ERR_UNSUPPORTED = 9, /* no kernel for this configuration (forced path not applicable) */
  FB_ERR_SCRATCH_LIMIT = 10 /* fb_born_bwd_static_scratch: backward needs more than its static scratch */
};

/* Element types. */
enum { FB_F32 = 0, FB_F16 = 1, FB_BF16 = 2 };

/* Kernel path selection (fb_attn_args.path). */
enum {
  FB_PATH_AUTO = 0,      /* tensor-core path when applicable, else the general path */
  FB_PATH_TCGEN05 = 1,   /* force the tcgen05/TMEM/TMA path (FB_ERR_UNSUPPORTED if not applicable) */
  FB_PATH_GENERAL = 2    /* force the general fp32-accumulating CUDA-core path */
};

typedef struct fb_attn_args {
  /* Problem shape. */
  int32_t batch, heads, seq_len, head_dim;
  /* Element type of q, k, v, dout, dq, dk, dv. */
  int32_t dtype;
  /* Element type of out (the forward output; the backward reads it back for delta).
   * Equal to dtype, or FB_F32: purified Born writes fp32 (flash_born.py:1102); a plain forward
   * whose output is one term of a sum of score families (complex phase, paired heads) writes
   * fp32 so the terms combine at full precision (ABI 4). */
  int32_t out_dtype;
  int32_t is_causal;
  int32_t window_size; /* 0 = no window; else i - j < window_size */
  float eps;           /* added after the row sum: Z = sum p + eps */
  float eps_base;      /* purified only: weight of the relu(raw)^2 floor */
  int32_t path;        /* FB_PATH_* */
  int32_t deterministic; /* 1: no floating-point atomics in the backward */

  const void* q;    int64_t q_stride[4];
  const void* k;    int64_t k_stride[4];
  const void* v;    int64_t v_stride[4];
  void* out;        int64_t out_stride[4];
  float* z; /* (B, H, T) contiguous */

  const float* scale; int32_t scale_numel; /* plain: scale; purified: gamma */
  const float* tau;   int32_t tau_numel;   /* purified only */

  const int32_t* doc_ids; int64_t doc_stride[2]; /* NULL = no document mask */

  /* Backward only. */
  const void* dout; int64_t dout_stride[4];
  void* dq;         int64_t dq_stride[4];
  void* dk;         int64_t dk_stride[4];
  void* dv;         int64_t dv_stride[4];
  float* dscale; /* accumulated, scale_numel elements */
  float* dtau;   /* accumulated, tau_numel elements (purified) */

  /* Backward: fb_bwd_workspace_size() bytes.  Forward: fb_fwd_workspace_size() bytes, which is
   * non-zero only with doc_ids on the tensor-core path (document spans used to skip tiles, and the
   * runs of equal ids that turn the document mask into one range per row). */
  void* workspace; size_t workspace_bytes;
} fb_attn_args;

/* Plain flash-Born forward: writes out and z. Replaces flash_born.py:475-513. */
FB_API int fb_born_fwd(const fb_attn_args* args, void* stream);

/* Plain flash-Born backward: writes dq, dk, dv; accumulates dscale.
 * Replaces flash_born.py:554-612 (dK/dV/dscale kernel + dQ kernel). */
FB_API int fb_born_bwd(const fb_attn_args* args, void* stream);

/* Purified (degree-4 thresholded) forward. Replaces flash_born.py:1110-1147. */
FB_API int fb_purified_born_fwd(const fb_attn_args* args, void* stream);

/* Purified backward: dq, dk, dv; accumulates dscale (d gamma) and dtau.
 * Replaces flash_born.py:1197-1262. */
FB_API int fb_purified_born_bwd(const fb_attn_args* args, void* stream);

/* Backward of one term of a sum of plain Born score families that share one normaliser
 * (ABI 4).  Complex-phase Born (layers/attention.py:717-730: p = relu(a s_re)^2 + relu(a s_im)^2,
 * s_im = <q, rot k>) and paired heads (layers/attention.py:591-626: a query row attends the keys
 * of both heads of its pair) are such sums; each term is one plain Born problem over its own
 * (q, k, v) views.  `out` and `z` are the WHOLE sum's forward output and Z (Z = sum over all terms
 * and keys of p + eps); dq, dk, dv receive this term's share of the gradients (the caller adds
 * the terms).  dscale / dtau are neither read nor written: the scale gradient of the sum is
 * (2 / scale_h) sum_{b,i} eps delta_i / Z_i with delta_i = dO_i . O_i, formed by the caller.
 * Same workspace as fb_born_bwd.  No single counterpart in the reference, whose complex-phase
 * and paired-heads paths are eager PyTorch (the lines cited above). */
FB_API int fb_born_bwd_term(const fb_attn_args* args, void* stream);

/* Glue of the families run as sums of plain Born terms (ABI 4); no counterpart in the reference,
 * whose complex-phase and paired-heads paths are eager PyTorch (layers/attention.py:717-730,
 * :591-626).
 *   fb_rotate_halves   dst = a + R b per row of head_dim = 2 h elements, R b = [-b_im | b_re]
 *                      (adjoint = 0: the key of the imaginary overlap <q, R k> = q_im.k_re - q_re.k_im)
 *                      or R^T b = [b_im | -b_re] (adjoint = 1: its gradient); a may be NULL; rows
 *                      contiguous, a / b / dst of one dtype
 *   fb_combine_terms   O = sum_t O_t Z_t / sum_t Z_t, Z = sum_t Z_t over n_terms (1..4) term outputs
 *                      O_t (B, H, T, D) fp32 contiguous (16-byte aligned) and Z_t (B, H, T) fp32
 *                      contiguous; O written as out_dtype through out_stride, Z through z_stride
 *   fb_delta_terms     part[b, h, c] = sum_t eps (dO . O) / Z over rows t of 64-row chunk c of
 *                      (b, h): the family's scale gradient is (2 / scale) times the sum of part
 *                      over the rows that scale entry serves (Z contiguous (B, H, T); part
 *                      (B, H, ceil(T / 64)) fp32) */
typedef struct fb_rot_args {
  int64_t rows;
  int32_t head_dim;
  int32_t dtype;
  int32_t adjoint;
  const void* a;
  const void* b;
  void* dst;
} fb_rot_args;

typedef struct fb_combine_args {
  int32_t batch, heads, seq_len, head_dim;
  int32_t n_terms;
  int32_t out_dtype;
  const float* o[4];
  const float* z[4];
  void* out;    int64_t out_stride[4];
  float* z_out; int64_t z_stride[3];
} fb_combine_args;

typedef struct fb_delta_args {
  int32_t batch, heads, seq_len, head_dim;
  int32_t dout_dtype, out_dtype;
  float eps;
  const void* dout; int64_t dout_stride[4];
  const void* out;  int64_t out_stride[4];
  const float* z;
  float* part;
} fb_delta_args;

FB_API int fb_rotate_halves(const fb_rot_args* args, void* stream);
FB_API int fb_combine_terms(const fb_combine_args* args, void* stream);
FB_API int fb_delta_terms(const fb_delta_args* args, void* stream);

/* ------------------------------------------------------------------------------------------
 * The layer's head epilogue (ABI version 4), _finalize_heads of the reference
 * (layers/attention.py:478-493) up to out_proj:
 *   r = y - tanh(alpha_h) (y . v) / (|v|^2 + eps) v      gated XSA (layers/mudd_and_gates.py:45-61),
 *                                                        when xsa_alpha is given
 *   g = 2 sigmoid(b_h + sum_k x[b, t, k] W[h, k])        input gate (mudd_and_gates.py:17-42), when
 *                                                        gate_x is given (else g = 1)
 *   Y[b, t, h hd + i] = g r_i                            heads merged for out_proj
 * o (the attention output) and v are (B, H, T, hd) with any 16-byte aligned strides (unit inner
 * stride); Y and dY are (B, T, H hd) contiguous; gate_x (B, T, gate_channels <= 8), gate_w
 * (H, gate_channels), gate_b and xsa_alpha (H) are fp32 contiguous; dtype FB_BF16 or FB_F32 for
 * o, v, Y and the gradients; hd 32, 64 or 128.  The backward writes grad_o and grad_v (B, H, T, hd)
 * contiguous and, per (b, t, h), dalpha = d/d alpha_h and du = d/d (gate pre-activation), whose
 * sums over rows (and products with gate_x) give the parameter gradients.
 * ------------------------------------------------------------------------------------------ */
typedef struct fb_heads_args {
  int32_t batch, heads, seq_len, head_dim;
  int32_t dtype;
  float eps;
  const void* o; int64_t o_stride[4];
  const void* v; int64_t v_stride[4];
  const float* xsa_alpha;
  const float* gate_x; int32_t gate_channels;
  const float* gate_w;
  const float* gate_b;
  void* y;          /* forward output */
  const void* dy;   /* backward input */
  void* grad_o;     /* backward outputs */
  void* grad_v;
  float* dalpha;
  float* du;
} fb_heads_args;

FB_API int fb_heads_epilogue_fwd(const fb_heads_args* args, void* stream);
FB_API int fb_heads_epilogue_bwd(const fb_heads_args* args, void* stream);

/* Plain flash-Born backward that allocates nothing and takes no workspace: its scratch is a
 * fixed FB_STATIC_SCRATCH_BYTES device array inside the library, for callers that cannot
 * allocate device memory (a host runtime with no device allocator of its own, or a step that
 * must not call cudaMalloc).  The array belongs to the library's device module: every GPU holds
 * it from the time the module loads there until exit (with CUDA's default lazy module loading,
 * the first launch of any of this library's kernels on that GPU; with CUDA_MODULE_LOADING=EAGER,
 * context creation), whether or not this entry point is called.
 * Same arguments and results as fb_born_bwd except workspace/workspace_bytes, which it ignores.
 * Returns FB_ERR_SCRATCH_LIMIT when fb_bwd_workspace_size() exceeds FB_STATIC_SCRATCH_BYTES, and
 * FB_ERR_ARG for purified arguments (tau != NULL): plain Born only.
 * The first successful call on a device looks up the array's address there; make it before any
 * stream capture.  All calls on a device share the array, which keeps the last call's contents
 * (each call rewrites what it reads): calls that overlap on the GPU race.
 * No counterpart in the reference (its kernels allocate through PyTorch). */
#define FB_STATIC_SCRATCH_BYTES (16u * 1024u * 1024u)
FB_API int fb_born_bwd_static_scratch(const fb_attn_args* args, void* stream);

/* Test hook, not for production use: the plain forward on the tensor-core path (FB_ERR_UNSUPPORTED
 * where that path does not apply) with every device-side wait bounded by wait_limit_us
 * microseconds instead of one second, and CTA 0's producer never requesting its first K tile.
 * The waits on that tile run into their bound, so the CTA takes the path a broken pipeline would:
 * it raises its abort flag, lets the copies and products already in flight land (each wait again
 * bounded), frees its tensor memory and returns, and the device status word reads FB_ERR_TIMEOUT
 * with the site of the first wait that gave up (fb_device_status).  Nothing faults, traps or
 * hangs; the context stays usable; this call's out and z are invalid.
 * No counterpart in the reference. */
FB_API int fb_test_born_fwd_timeout(const fb_attn_args* args, void* stream, uint32_t wait_limit_us);

/* Bytes of device workspace the backward needs for these arguments (0 allowed for none).
 * A non-NULL tau marks purified arguments here and in fb_select_path.
 * The reference allocates the equivalent scratch implicitly (delta is recomputed per tile). */
FB_API size_t fb_bwd_workspace_size(const fb_attn_args* args);

/* Bytes of device workspace the forward needs for these arguments: 0 without doc_ids; with them,
 * room for the per-64-row-block document spans that let the tensor-core kernels skip tiles with
 * no same-document pair, and for the per-position runs of equal ids (about batch * seq_len * 8
 * bytes) with which rows whose ids never decrease mask by one range.  ABI version 2.  No counterpart in the reference (its forward visits
 * every causal tile and masks, flash_born.py:169-178). */
FB_API size_t fb_fwd_workspace_size(const fb_attn_args* args);

/* Which path fb_*_fwd / fb_*_bwd would take for these arguments: FB_PATH_TCGEN05 or
 * FB_PATH_GENERAL, or a negative FB_ERR_* if the arguments are invalid. `backward` selects
 * the backward kernels. Replaces get_flash_born_launch_meta (flash_born.py:31-65) as the
 * host-visible tile policy. */
FB_API int fb_select_path(const fb_attn_args* args, int backward);

/* Number of kernel launches the last successful fb_* call on this host thread enqueued. */
FB_API int fb_last_launch_count(void);

/* Reads (and clears) the device status word of the current device: FB_OK or FB_ERR_TIMEOUT.
 * Synchronises `stream`. `detail` (may be NULL) receives the site code of the first failure. */
FB_API int fb_device_status(void* stream, int32_t* detail);

/* Human-readable message for a status code. */
FB_API const char* fb_strerror(int status);

/* The last CUDA runtime error string seen by the library on this host thread. */
FB_API const char* fb_last_cuda_error(void);

/* FB_ABI_VERSION of the built library. */
FB_API int fb_abi_version(void);

/* ------------------------------------------------------------------------------------------
 * The attention layer's operand prologue (ABI version 3).  The reference builds Q, K, V with a
 * chain of PyTorch ops (layers/attention.py:512-516 reshape / transpose / contiguous of the fused
 * projection, :573-589 apply_unitary_rope then l2_normalize, functional.py:59-121); these kernels
 * do it in one pass each way.
 *
 *   forward   Q = l2n(rope(qkv[..., 0:D])), K = l2n(rope(qkv[..., D:2D])), V = qkv[..., 2D:3D],
 *             each written (B, H, T, hd) contiguous; D = H hd
 *   backward  dqkv from dQ, dK, dV (B, H, T, hd) contiguous and qkv
 *   rope      per head, element i < hd/2 and its partner i + hd/2 turn by angle (t, i):
 *             (u_i, u_{i+hd/2}) -> (u_i cos - u_{i+hd/2} sin, u_i sin + u_{i+hd/2} cos)
 *   l2n       y = y / sqrt(sum y^2 + eps)
 * qkv is (B, T, 3 D) contiguous; cos / sin are (T, hd/2) contiguous fp32; hd is 64 or 128;
 * dtype FB_BF16 or FB_F32 for qkv and every (B, H, T, hd) tensor; arithmetic in fp32.
 * ------------------------------------------------------------------------------------------ */
typedef struct fb_qkv_args {
  int32_t batch, seq_len, heads, head_dim;
  int32_t dtype;
  float eps;
  const void* qkv;
  const float* cos;
  const float* sin;
  void* q; /* forward: outputs; backward: the incoming gradients dQ, dK, dV */
  void* k;
  void* v;
  void* dqkv; /* backward output */
} fb_qkv_args;

FB_API int fb_qkv_prologue_fwd(const fb_qkv_args* args, void* stream);
FB_API int fb_qkv_prologue_bwd(const fb_qkv_args* args, void* stream);

/* Row L2 normalisation, the layer's psi = l2_normalize(x) (functional.py:59-81):
 *   forward   y = x / sqrt(sum x^2 + eps) over each row of `cols` elements
 *   backward  dx = r (dy - y (y . dy)),  r = 1 / sqrt(sum x^2 + eps)
 * Rows contiguous (row stride = cols); cols a multiple of 8 (bf16) or 4 (fp32); pointers 16-byte
 * aligned. */
typedef struct fb_rows_args {
  int64_t rows;
  int32_t cols;
  int32_t dtype;
  float eps;
  const void* x;
  void* y;
  const void* dy;
  void* dx;
} fb_rows_args;

FB_API int fb_l2norm_rows_fwd(const fb_rows_args* args, void* stream);
FB_API int fb_l2norm_rows_bwd(const fb_rows_args* args, void* stream);

/* ------------------------------------------------------------------------------------------
 * The GPT training loss (ABI version 4): mean cross-entropy over bf16 logits, replacing
 * F.cross_entropy(logits.reshape(-1, V), targets) of the reference's GPTs
 * (models/born_gpt.py:1291), which under bf16 autocast runs over an fp32 copy of the logits.
 *   forward   lse[r] = log sum_c exp(x[r, c]),  loss[r] = lse[r] - x[r, targets[r]]
 *             (the caller averages loss over the rows)
 *   backward  grad[r, c] = (exp(x[r, c] - lse[r]) - [c == targets[r]]) * gscale[0] / rows
 * logits and grad are bf16 rows of `vocab` elements `ld` apart (vocab and ld multiples of 8,
 * pointers 16-byte aligned); columns holding -inf take no probability.  targets are int64; a
 * target outside [0, vocab) gives a NaN loss.  lse and loss are fp32 (rows); gscale is a device
 * fp32 scalar (the incoming gradient of the mean loss).
 * ------------------------------------------------------------------------------------------ */
typedef struct fb_xent_args {
  int64_t rows;
  int32_t vocab;
  int64_t ld;
  const void* logits;
  const int64_t* targets;
  float* lse;
  float* loss;         /* forward output */
  void* grad;          /* backward output */
  const float* gscale; /* backward input */
} fb_xent_args;

FB_API int fb_xent_fwd(const fb_xent_args* args, void* stream);
FB_API int fb_xent_bwd(const fb_xent_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHBORN_B200_H_ */

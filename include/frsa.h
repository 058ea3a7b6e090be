/*
 * frsa.h — C ABI of the B200 (sm_100a) fused 2D-RoPE scaled-dot-product
 * attention, forward and backward.
 *
 * The reference (v1kstrand/triton_fused_rope_flash_attn, file "fa_rope_full .py")
 * has no native ABI: its Python autograd wrapper launches Triton kernels
 * directly. Each entry point below replaces one group of those launches; the
 * host mirror (triton_fused_rope_flash_attn_b200.TritonAttention) calls them
 * through ctypes with torch-allocated device buffers.
 *
 * Conventions
 *   - All tensor pointers are device pointers. q, k, v are [B, H, N, D] in the
 *     I/O dtype with unit d stride (contiguous unless *_strides say otherwise);
 *     o, d_o, dq, dk, dv are contiguous [B, H, N, D]; lse and delta are
 *     contiguous fp32 [B, H, N]; cosp/sinp are contiguous fp32 [n_pos, D/2].
 *   - Token t uses table row t - has_cls; token 0 is not rotated when has_cls.
 *   - scale multiplies the logits (the reference uses 1/sqrt(D)).
 *   - lse receives max + ln(sum) of the scaled logits per query row, the
 *     quantity the reference stores in M (fa_rope_full .py:309).
 *   - Launches are asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *     default stream). Entry points never allocate device memory: scratch is
 *     passed in by the caller.
 *   - Return value 0 = launched; otherwise an FRSA_ERR_* code, nothing launched.
 *     A CUDA error already pending on the calling thread (from the caller's
 *     own earlier work) is reported as FRSA_ERR_LAUNCH and left pending.
 *   - Thread-safe; no global state except the device status word below.
 */
#ifndef FRSA_H_
#define FRSA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FRSA_ABI_VERSION 2

enum frsa_dtype {
  FRSA_DTYPE_BF16 = 0,
  FRSA_DTYPE_F16 = 1,
  FRSA_DTYPE_F32 = 2
};

enum frsa_status {
  FRSA_OK = 0,
  FRSA_ERR_NULL_ARG = 1,        /* a required pointer is NULL */
  FRSA_ERR_BAD_SHAPE = 2,       /* B, H, N or D out of range, or N inconsistent with n_pos/has_cls */
  FRSA_ERR_UNSUPPORTED_D = 3,   /* D % 8 != 0 or D > 128 */
  FRSA_ERR_UNSUPPORTED_DTYPE = 4,
  FRSA_ERR_MISALIGNED = 5,      /* a pointer is not 16-byte aligned */
  FRSA_ERR_LAUNCH = 6,          /* a CUDA launch or tensor-map encode failed */
  FRSA_ERR_DEVICE_TIMEOUT = 7,  /* a kernel gave up on a bounded wait (see frsa_query_status) */
  FRSA_ERR_NO_DEVICE = 8,       /* the current device is not sm_100 */
  FRSA_ERR_WORKSPACE = 9,       /* the backward workspace is missing or too small */
  FRSA_ERR_SCRATCH_LIMIT = 10   /* B*H*N*D exceeds frsa_bwd_noalloc_max_elements() */
};

typedef struct frsa_attn_args {
  /* forward inputs / outputs */
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  /* backward inputs / outputs (ignored by frsa_fwd) */
  const void* d_o;
  void* dq;
  void* dk;
  void* dv;
  float* delta;       /* optional fp32 [B, H, N]: receives rowsum(dO * O) when non-NULL */
  void* workspace;    /* fp32 scratch of frsa_bwd_workspace_bytes() bytes, or NULL when that is 0 */
  size_t workspace_bytes;
  /* RoPE pair tables */
  const float* cosp;
  const float* sinp;
  /* shape */
  int64_t B, H, N, D, n_pos;
  int32_t has_cls;
  int32_t io_dtype;       /* enum frsa_dtype; must equal compute_dtype in this ABI version */
  int32_t compute_dtype;  /* enum frsa_dtype: BF16 or F16; F32 = float32 tensors with
                             TF32 tensor-core products (frsa_bwd: D <= 64, and a Delta
                             workspace of B*H*N floats unless `delta` is given) */
  float scale;
  /* Optional element strides (b, h, n) of q, k and v; the d stride is 1. All
   * zero = contiguous [B, H, N, D]. Non-zero strides must be multiples of 16
   * bytes (e.g. the q, k, v views of a [B, N, 3, H, D] projection output), and
   * the pointers 16-byte aligned. Other tensors are always contiguous. */
  int64_t q_strides[3];
  int64_t k_strides[3];
  int64_t v_strides[3];
  /* FRSA_FLAG_* bits. */
  int32_t flags;
} frsa_attn_args;

/* q and k arrive already rotated (e.g. by frsa_qkv_rope, which applies the
 * RoPE in the projection's epilogue): the kernels skip every rotation, and
 * frsa_bwd returns dq and dk with respect to the given q and k (no R^T).
 * cosp/sinp may then be NULL and n_pos is not checked. No counterpart in the
 * reference, whose kernels always rotate. */
#define FRSA_FLAG_NO_ROPE 1

/* Forward: O = softmax(R(Q) R(K)^T * scale) V and lse.
 * Replaces the _attn_fwd launch of TritonAttention.forward
 * (fa_rope_full .py:1036-1057; kernel fa_rope_full .py:91-315). */
int frsa_fwd(const frsa_attn_args* args, void* stream);

/* Backward: dQ, dK, dV from d_o, o, lse (and q, k, v, tables).
 * Replaces the three launches of TritonAttention.backward
 * (_attn_bwd_preprocess fa_rope_full .py:1076-1082, _attn_bwd_dk_dv_rope
 * fa_rope_full .py:1084-1107, _attn_bwd_dq_rope fa_rope_full .py:1109-1136)
 * with one persistent kernel (N <= 256 and D <= 64), or otherwise with a
 * counter clear, a row pass (rotated Q and K, Delta) and one persistent
 * key-tile kernel whose dQ is reduced over key tiles in a fixed order. Results are bitwise reproducible
 * from call to call in both cases. */
int frsa_bwd(const frsa_attn_args* args, void* stream);

/* Bytes of workspace frsa_bwd needs for this shape: 0 when the whole head fits
 * one CTA (N <= 256, D <= 64, 16-bit), else, for 16-bit compute, with
 * T = ceil(N/128) key tiles and S = min(T, 8) partial-dQ slots,
 *   S * B*H*N*D floats (partial dQ sums)
 * + 4 * ((B*H*T*(1 + S) + 4) & ~3) bytes (arrival and slot counters, a claim ticket)
 * + 2 * B*H*N*D 16-bit values (the rotated Q and K)
 * + B*H*N floats (Delta rows), the last term only when args->delta is NULL;
 * for F32 compute, B*H*N floats of Delta when args->delta is NULL.
 * ABI version 2 (version 1 asked for B*H*N*(D+1) floats in every case).
 * No reference counterpart: the reference's dQ kernel (fa_rope_full
 * .py:708-1009) recomputes S and dP instead of reducing over key tiles. */
size_t frsa_bwd_workspace_bytes(const frsa_attn_args* args);

/* Backward pass that allocates nothing, for callers that cannot call
 * cudaMalloc: plugin hosts that only hand over input and output buffers,
 * runtimes whose device memory is fully carved up in advance, or loops that
 * must avoid cudaMalloc/cudaFree because those can synchronise the device.
 * Same arguments as frsa_bwd, but `workspace` is ignored and only 16-bit
 * compute is accepted (F32 returns FRSA_ERR_UNSUPPORTED_DTYPE). Every shape
 * runs the general key-tile kernel with the ordered dQ reduction, whose f32
 * running sums and turn counters live in a fixed array inside the library
 * (20 MiB per device, kept until the process exits), so B*H*N*D must not
 * exceed frsa_bwd_noalloc_max_elements() (else FRSA_ERR_SCRATCH_LIMIT,
 * nothing launched). Results agree with frsa_bwd's to rounding (bitwise for
 * N > 256 or D > 64, where frsa_bwd runs the same kernel). The first call on a
 * device looks up that array's address (make it before any stream capture).
 * All calls on a device share the array: each clears the counters it uses,
 * and calls that run concurrently on the GPU race, so order them on one
 * stream. No counterpart in the reference. */
int frsa_bwd_noalloc(const frsa_attn_args* args, void* stream);

/* Largest B*H*N*D frsa_bwd_noalloc accepts (4 Mi elements). No counterpart in
 * the reference. */
size_t frsa_bwd_noalloc_max_elements(void);

/* Message for an FRSA_ERR_* code (static storage). */
const char* frsa_strerror(int code);

/* Detail (CUDA error string and call) of the last FRSA_ERR_LAUNCH returned on
 * the calling host thread; "" if none. No reference counterpart. */
const char* frsa_last_error_detail(void);

/* Synchronizes the current device, returns FRSA_ERR_DEVICE_TIMEOUT if any
 * kernel recorded a bounded-wait timeout since the last call (and clears it),
 * FRSA_ERR_LAUNCH on a sticky CUDA error, else FRSA_OK. */
int frsa_query_status(void);

/* QKV projection with the 2D RoPE applied in its epilogue: for x [B*N, C]
 * (token rows), the nn.Linear weight w [3C, C] and bias [3C] (fp32),
 *   q = R(x w[0:C]^T + b[0:C]), k = R(x w[C:2C]^T + b[C:2C]), v = x w[2C:]^T + b[2C:],
 * each written as [B, H, N, D] (D = C / H) in `dtype`; R rotates token n with
 * table row n - has_cls and leaves the CLS token as is. Attention over these
 * q, k then needs no further rotation (use identity tables). Requires
 * C % 128 == 0 and D % 32 == 0 (else FRSA_ERR_UNSUPPORTED_D).
 * No counterpart in the reference: it fuses the projection that precedes the
 * reference's kernel in timm's attention block (reference README:156-159). */
typedef struct frsa_qkv_args {
  const void* x;
  const void* w;
  const float* bias;
  const float* cosp;
  const float* sinp;
  void* q;
  void* k;
  void* v;
  int64_t B, N, C, H, n_pos;
  int32_t has_cls;
  int32_t dtype;      /* enum frsa_dtype: BF16 or F16 */
} frsa_qkv_args;

int frsa_qkv_rope(const frsa_qkv_args* args, void* stream);

/* Backward of frsa_qkv_rope's epilogue: from the gradients of its outputs
 * dq, dk, dv ([B, H, N, D] each, `dtype`, contiguous; dq and dk with respect
 * to the rotated q and k), writes dqkv [B*N, 3C] (`dtype`), the gradient of
 * the projection output x w^T + b: R^T applied to the q and k parts in f32,
 * one rounding, heads merged back into channels. Then dx = dqkv w,
 * dw = dqkv^T x and db = the column sums of dqkv. Same shape rules as
 * frsa_qkv_rope (C % 128 == 0, D % 32 == 0). No counterpart in the reference
 * (see frsa_qkv_rope). */
typedef struct frsa_qkv_bwd_args {
  const void* dq;
  const void* dk;
  const void* dv;
  const float* cosp;
  const float* sinp;
  void* dqkv;
  int64_t B, N, C, H, n_pos;
  int32_t has_cls;
  int32_t dtype;      /* enum frsa_dtype: BF16 or F16 */
} frsa_qkv_bwd_args;

int frsa_qkv_rope_bwd(const frsa_qkv_bwd_args* args, void* stream);

/* f32 inputs under 16-bit compute (the reference converts f32 loads to the
 * compute type, fa_rope_full .py:168-174, 240-246). frsa_convert_in reads q,
 * k, v (f32, contiguous [B, H, N, D]) and writes q_out = R(q), k_out = R(k)
 * and v_out in `dtype` (BF16 or F16), rotated in f32 and rounded once, so
 * that frsa_fwd / frsa_bwd then run with FRSA_FLAG_NO_ROPE. frsa_convert_out
 * is its backward: q, k, v are the 16-bit gradients with respect to q_out,
 * k_out, v_out, and q_out, k_out, v_out receive dq = R^T dq^, dk = R^T dk^
 * and dv in f32. Rotation as in frsa_fwd (table row n - has_cls, the CLS
 * token untouched). D % 8 == 0, every pointer 16-byte aligned. No direct
 * counterpart in the reference (its kernels convert while loading). */
typedef struct frsa_convert_args {
  const void* q;
  const void* k;
  const void* v;
  void* q_out;
  void* k_out;
  void* v_out;
  const float* cosp;
  const float* sinp;
  int64_t B, H, N, D, n_pos;
  int32_t has_cls;
  int32_t dtype;      /* enum frsa_dtype of the 16-bit side: BF16 or F16 */
} frsa_convert_args;

int frsa_convert_in(const frsa_convert_args* args, void* stream);
int frsa_convert_out(const frsa_convert_args* args, void* stream);

/* FRSA_ABI_VERSION of the loaded library. */
int frsa_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FRSA_H_ */

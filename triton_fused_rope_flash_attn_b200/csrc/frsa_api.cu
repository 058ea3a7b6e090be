// C ABI (include/frsa.h): argument validation, TMA tensor-map encoding and
// dispatch to the sm_100a kernels. This is the library's only translation
// unit; the kernel files are included so that the device status word is one
// symbol without relocatable device code.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/frsa.h"
#include "frsa_internal.h"
#include "frsa_ptx.cuh"

#include "frsa_bwd.cu"
#include "frsa_bwd_small.cu"
#include "frsa_fwd.cu"
#include "frsa_fwd_small.cu"
#include "frsa_tf32.cu"
#include "frsa_qkv.cu"
#include "frsa_convert.cu"

namespace frsa {

int device_sm_count() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

cudaError_t set_max_dynamic_smem_once(const void* kernel, size_t bytes) {
  // (kernel, device) pairs already configured; the library has ~20 kernels.
  struct Entry { const void* k; int dev; size_t bytes; };
  static Entry done[256];
  static int ndone = 0;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < ndone; ++i)
    if (done[i].k == kernel && done[i].dev == dev && done[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes));
  if (e == cudaSuccess && ndone < 256) done[ndone++] = Entry{kernel, dev, bytes};
  return e;
}

}  // namespace frsa

namespace {

using frsa::kTile;

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Is the current device an sm_100 part? Cached per device ordinal. Also makes
// the device's primary context current on this host thread: the tensor-map
// encoder is a driver call and needs it, and a thread that has not touched the
// runtime yet (autograd's backward worker, a user thread) may have none.
bool device_is_sm100() {
  static int cache[64];  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaSetDevice(dev) != cudaSuccess) return false;
  if (dev < 0 || dev >= 64) return false;
  if (cache[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cache[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  return cache[dev] == 1;
}

thread_local int g_last_encode_result = 0;
// Detail of the last FRSA_ERR_LAUNCH on this host thread.
thread_local char g_last_detail[256] = "";

// 4-D map over a [B, H, N, D] tensor: dims {D, N, H, B}; `st` gives the
// n, h, b strides in elements (nullptr: contiguous). Box {64, 128, 1, 1} for
// 16-bit tensors, {32, 128, 1, 1} for float32 (s.f32): 128 bytes per row
// either way, 128-byte swizzle, zero fill outside the tensor. atom32: for
// float32 operands read MN-major by kind::tf32 products, the 128-byte swizzle
// with 32-byte atoms that such operands need.
bool encode_map(CUtensorMap* m, const void* base, const frsa::LaunchShape& s,
                bool atom32 = false, const int64_t* st = nullptr) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t elt = s.f32 ? 4 : 2;
  const cuuint64_t H = static_cast<cuuint64_t>(s.H), B = static_cast<cuuint64_t>(s.BH / s.H);
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(s.D), static_cast<cuuint64_t>(s.N), H, B};
  const cuuint64_t sn = st ? static_cast<cuuint64_t>(st[2]) : static_cast<cuuint64_t>(s.D);
  const cuuint64_t sh = st ? static_cast<cuuint64_t>(st[1]) : sn * s.N;
  const cuuint64_t sb = st ? static_cast<cuuint64_t>(st[0]) : sh * H;
  const cuuint64_t strides[3] = {sn * elt, sh * elt, sb * elt};
  const cuuint32_t box[4] = {s.f32 ? 32u : 64u, 128, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = s.f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : s.bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(m, dt,
                        4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) g_last_encode_result = static_cast<int>(r);
  return r == CUDA_SUCCESS;
}

// 3-D f32 map {D, N, planes} over contiguous [planes, N, D] rows, box
// {32, 128, 1}, 128-byte swizzle (the general backward's partial-dQ slots).
bool encode_map_f32_3d(CUtensorMap* m, const float* base, long long planes, int N, int D) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N),
                              static_cast<cuuint64_t>(planes)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 4,
                                 static_cast<cuuint64_t>(D) * N * 4};
  const cuuint32_t box[3] = {32, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) g_last_encode_result = static_cast<int>(r);
  return r == CUDA_SUCCESS;
}

// 2-D map over a contiguous [rows, cols] 16-bit matrix, box {64, 128}.
bool encode_map_2d(CUtensorMap* m, const void* base, long long rows, long long cols, bool bf16) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) g_last_encode_result = static_cast<int>(r);
  return r == CUDA_SUCCESS;
}


int launch_error(const char* where, cudaError_t e) {
  if (e == cudaSuccess)
    snprintf(g_last_detail, sizeof(g_last_detail), "%s: tensor-map encode failed (CUresult %d)",
             where, g_last_encode_result);
  else
    snprintf(g_last_detail, sizeof(g_last_detail), "%s: %s (%d)", where, cudaGetErrorString(e),
             static_cast<int>(e));
  return FRSA_ERR_LAUNCH;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Caller strides of a q/k/v tensor, or nullptr when it is contiguous.
const int64_t* strides_of(const int64_t* st) {
  return (st[0] == 0 && st[1] == 0 && st[2] == 0) ? nullptr : st;
}

// f32 map {D, N, nslot * BH} over the general backward's partial-dQ slots,
// box {32, 128, 1}, 128-byte swizzle.
bool encode_part_map(CUtensorMap* m, const float* part, const frsa::LaunchShape& s, int nslot) {
  return encode_map_f32_3d(m, part, static_cast<long long>(s.BH) * nslot, s.N, s.D);
}

// A CUDA error already pending on this host thread (left by the caller's own
// earlier work) is reported, not cleared: nothing is launched, the error stays
// pending for its owner, and the detail string names it.
int pending_error(const char* where) {
  const cudaError_t e = cudaPeekAtLastError();
  if (e == cudaSuccess) return FRSA_OK;
  snprintf(g_last_detail, sizeof(g_last_detail),
           "%s: a CUDA error was already pending before this call: %s (%d)", where,
           cudaGetErrorString(e), static_cast<int>(e));
  return FRSA_ERR_LAUNCH;
}

int validate_common(const frsa_attn_args* a, frsa::LaunchShape* s) {
  if (!a) return FRSA_ERR_NULL_ARG;
  const bool rope = (a->flags & FRSA_FLAG_NO_ROPE) == 0;
  if (a->flags & ~FRSA_FLAG_NO_ROPE) return FRSA_ERR_BAD_SHAPE;
  if (!a->q || !a->k || !a->v || (rope && (!a->cosp || !a->sinp))) return FRSA_ERR_NULL_ARG;
  if (a->B < 1 || a->H < 1 || a->N < 1 || a->D < 1) return FRSA_ERR_BAD_SHAPE;
  if (a->has_cls != 0 && a->has_cls != 1) return FRSA_ERR_BAD_SHAPE;
  if (a->D % 8 != 0 || a->D > 128) return FRSA_ERR_UNSUPPORTED_D;
  if (rope && a->N - a->has_cls > a->n_pos) return FRSA_ERR_BAD_SHAPE;  // table must cover every token
  const long long BH = static_cast<long long>(a->B) * a->H;
  const long long nqt = (a->N + kTile - 1) / kTile;
  if (BH * nqt > 0x7FFFFFFFLL || a->N > (1LL << 30)) return FRSA_ERR_BAD_SHAPE;
  if (a->io_dtype != a->compute_dtype) return FRSA_ERR_UNSUPPORTED_DTYPE;
  if (a->compute_dtype != FRSA_DTYPE_BF16 && a->compute_dtype != FRSA_DTYPE_F16 &&
      a->compute_dtype != FRSA_DTYPE_F32)
    return FRSA_ERR_UNSUPPORTED_DTYPE;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) ||
      (rope && (!aligned16(a->cosp) || !aligned16(a->sinp))))
    return FRSA_ERR_MISALIGNED;
  const int64_t elt = a->compute_dtype == FRSA_DTYPE_F32 ? 4 : 2;
  for (const int64_t* st : {a->q_strides, a->k_strides, a->v_strides}) {
    if (st[0] == 0 && st[1] == 0 && st[2] == 0) continue;
    for (int d = 0; d < 3; ++d)
      if (st[d] < 1 || (st[d] * elt) % 16 != 0 || st[d] * elt >= (int64_t(1) << 40))
        return FRSA_ERR_MISALIGNED;
  }
  s->BH = static_cast<int>(BH);
  s->H = static_cast<int>(a->H);
  s->N = static_cast<int>(a->N);
  s->D = static_cast<int>(a->D);
  s->has_cls = rope ? a->has_cls : -1;   // < 0: the kernels rotate nothing
  s->scale = a->scale;
  s->bf16 = a->compute_dtype == FRSA_DTYPE_BF16;
  s->f32 = a->compute_dtype == FRSA_DTYPE_F32;
  return FRSA_OK;
}

// Workspace of the general 16-bit backward: the f32 partial dQ sums (S slots
// of BH*N*D floats, S = min(key tiles, 8)), the counters and claim ticket,
// the rotated Q and K (BH*N*D 16-bit values each) and, unless the caller
// passes `delta`, the Delta rows (BH*N floats).
size_t general_bwd_workspace_bytes(const frsa::LaunchShape& s, bool caller_delta) {
  const size_t rows = static_cast<size_t>(s.BH) * s.N;
  const int S = frsa::bwd_slots(s);
  return S * rows * s.D * sizeof(float) + frsa::bwd_counter_ints(s, S) * sizeof(int) +
         2 * rows * s.D * 2 + (caller_delta ? 0 : rows * sizeof(float));
}

// float32 backward (TF32 tensor cores), D <= 64.
int bwd_f32(const frsa_attn_args* a, const frsa::LaunchShape& s, void* stream) {
  if (!frsa::tf32_bwd_supported(s)) return FRSA_ERR_UNSUPPORTED_D;
  if (!a->o || !a->lse || !a->d_o || !a->dq || !a->dk || !a->dv) return FRSA_ERR_NULL_ARG;
  if (!aligned16(a->o) || !aligned16(a->d_o) || !aligned16(a->dq) || !aligned16(a->dk) ||
      !aligned16(a->dv) || !aligned16(a->lse))
    return FRSA_ERR_MISALIGNED;
  float* delta = a->delta;
  if (delta == nullptr) {
    const size_t need = static_cast<size_t>(s.BH) * s.N * sizeof(float);
    if (!a->workspace || a->workspace_bytes < need) return FRSA_ERR_WORKSPACE;
    delta = static_cast<float*>(a->workspace);
  }
  if (!aligned16(delta)) return FRSA_ERR_MISALIGNED;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  if (const int rc = pending_error("frsa_bwd"); rc != FRSA_OK) return rc;
  CUtensorMap maps[7];   // q16, q32, k16, k32, v16, do16, do32
  const int64_t *sq = strides_of(a->q_strides), *sk = strides_of(a->k_strides),
                *sv = strides_of(a->v_strides);
  if (!encode_map(&maps[0], a->q, s, false, sq) || !encode_map(&maps[1], a->q, s, true, sq) ||
      !encode_map(&maps[2], a->k, s, false, sk) || !encode_map(&maps[3], a->k, s, true, sk) ||
      !encode_map(&maps[4], a->v, s, false, sv) || !encode_map(&maps[5], a->d_o, s) ||
      !encode_map(&maps[6], a->d_o, s, true))
    return launch_error("frsa_bwd", cudaSuccess);
  const cudaError_t e = frsa::launch_bwd_tf32(
      s, maps, static_cast<const float*>(a->o), static_cast<const float*>(a->d_o), a->lse, delta,
      a->cosp, a->sinp, static_cast<float*>(a->dq), static_cast<float*>(a->dk),
      static_cast<float*>(a->dv), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FRSA_OK : launch_error("frsa_bwd", e);
}

}  // namespace

extern "C" {

int frsa_abi_version(void) { return FRSA_ABI_VERSION; }

const char* frsa_strerror(int code) {
  switch (code) {
    case FRSA_OK: return "ok";
    case FRSA_ERR_NULL_ARG: return "frsa: a required pointer is NULL";
    case FRSA_ERR_BAD_SHAPE: return "frsa: bad shape (B, H, N, D, has_cls or table size)";
    case FRSA_ERR_UNSUPPORTED_D: return "frsa: head dim must be a multiple of 8 and at most 128";
    case FRSA_ERR_UNSUPPORTED_DTYPE: return "frsa: unsupported dtype combination";
    case FRSA_ERR_MISALIGNED: return "frsa: a tensor pointer is not 16-byte aligned";
    case FRSA_ERR_LAUNCH: return "frsa: CUDA launch or tensor-map encode failed";
    case FRSA_ERR_DEVICE_TIMEOUT: return "frsa: a kernel timed out on a bounded wait";
    case FRSA_ERR_NO_DEVICE: return "frsa: the current CUDA device is not sm_100";
    case FRSA_ERR_WORKSPACE: return "frsa: backward workspace missing or too small";
    case FRSA_ERR_SCRATCH_LIMIT:
      return "frsa: B*H*N*D exceeds the built-in scratch of frsa_bwd_noalloc "
             "(see frsa_bwd_noalloc_max_elements)";
    default: return "frsa: unknown error";
  }
}

size_t frsa_bwd_workspace_bytes(const frsa_attn_args* a) {
  frsa::LaunchShape s;
  if (validate_common(a, &s) != FRSA_OK) return 0;
  if (s.f32)   // Delta scratch of the float32 backward (unless args->delta is given)
    return (frsa::tf32_bwd_supported(s) && a->delta == nullptr)
               ? static_cast<size_t>(s.BH) * s.N * sizeof(float) : 0;
  if (!frsa::bwd_needs_workspace(s)) return 0;
  return general_bwd_workspace_bytes(s, a->delta != nullptr);
}

int frsa_fwd(const frsa_attn_args* a, void* stream) {
  frsa::LaunchShape s;
  int rc = validate_common(a, &s);
  if (rc != FRSA_OK) return rc;
  if (!a->o || !a->lse) return FRSA_ERR_NULL_ARG;
  if (!aligned16(a->o) || !aligned16(a->lse)) return FRSA_ERR_MISALIGNED;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  if ((rc = pending_error("frsa_fwd")) != FRSA_OK) return rc;
  CUtensorMap tq, tk, tv, to;
  if (!encode_map(&tq, a->q, s, false, strides_of(a->q_strides)) ||
      !encode_map(&tk, a->k, s, false, strides_of(a->k_strides)) ||
      !encode_map(&tv, a->v, s, /*atom32=*/s.f32, strides_of(a->v_strides)) ||
      !encode_map(&to, a->o, s))
    return launch_error("frsa_fwd", cudaSuccess);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      s.f32 ? frsa::launch_fwd_tf32(s, tq, tk, tv, a->cosp, a->sinp, static_cast<float*>(a->o),
                                    a->lse, st)
            : frsa::launch_fwd(s, tq, tk, tv, to, a->cosp, a->sinp, a->o, a->lse, st);
  return e == cudaSuccess ? FRSA_OK : launch_error("frsa_fwd", e);
}

int frsa_bwd(const frsa_attn_args* a, void* stream) {
  frsa::LaunchShape s;
  int rc = validate_common(a, &s);
  if (rc != FRSA_OK) return rc;
  if (s.f32) return bwd_f32(a, s, stream);
  if (!a->o || !a->lse || !a->d_o || !a->dq || !a->dk || !a->dv)
    return FRSA_ERR_NULL_ARG;
  if (!aligned16(a->o) || !aligned16(a->d_o) || !aligned16(a->dq) || !aligned16(a->dk) ||
      !aligned16(a->dv) || !aligned16(a->lse))
    return FRSA_ERR_MISALIGNED;
  const bool general = frsa::bwd_needs_workspace(s);
  if (general) {
    if (!a->workspace || a->workspace_bytes < general_bwd_workspace_bytes(s, a->delta != nullptr))
      return FRSA_ERR_WORKSPACE;
    if (!aligned16(a->workspace)) return FRSA_ERR_MISALIGNED;
  }
  if (a->delta && !aligned16(a->delta)) return FRSA_ERR_MISALIGNED;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  if ((rc = pending_error("frsa_bwd")) != FRSA_OK) return rc;
  CUtensorMap tq, tk, tv, tdo, to, tgrads[3];
  if (!encode_map(&tq, a->q, s, false, strides_of(a->q_strides)) ||
      !encode_map(&tk, a->k, s, false, strides_of(a->k_strides)) ||
      !encode_map(&tv, a->v, s, false, strides_of(a->v_strides)) ||
      !encode_map(&tdo, a->d_o, s) || !encode_map(&to, a->o, s))
    return launch_error("frsa_bwd", cudaSuccess);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (!general) {
    if (!encode_map(&tgrads[0], a->dq, s) || !encode_map(&tgrads[1], a->dk, s) ||
        !encode_map(&tgrads[2], a->dv, s))
      return launch_error("frsa_bwd", cudaSuccess);
    e = frsa::launch_bwd_small(s, tq, tk, tv, tdo, to, tgrads, a->o, a->lse, a->delta, a->cosp,
                               a->sinp, a->dq, a->dk, a->dv, st);
  } else {
    const size_t rows = static_cast<size_t>(s.BH) * s.N;
    const int S = frsa::bwd_slots(s);
    float* part = static_cast<float*>(a->workspace);
    int* counters = reinterpret_cast<int*>(part + S * rows * s.D);
    uint16_t* q_rot = reinterpret_cast<uint16_t*>(counters + frsa::bwd_counter_ints(s, S));
    uint16_t* k_rot = q_rot + rows * s.D;
    float* delta_rows = a->delta ? a->delta : reinterpret_cast<float*>(k_rot + rows * s.D);
    frsa::QkRotation rot;
    rot.q = a->q;
    rot.k = a->k;
    const int64_t* sq = strides_of(a->q_strides);
    const int64_t* sk = strides_of(a->k_strides);
    const long long cn = s.D, ch = static_cast<long long>(s.D) * s.N,
                    cb = static_cast<long long>(s.D) * s.N * s.H;
    for (int d = 0; d < 3; ++d) {
      const long long dflt = d == 0 ? cb : d == 1 ? ch : cn;
      rot.q_strides[d] = sq ? sq[d] : dflt;
      rot.k_strides[d] = sk ? sk[d] : dflt;
    }
    rot.q_rot = q_rot;
    rot.k_rot = k_rot;
    CUtensorMap tpart;
    if (!encode_map(&tq, q_rot, s) || !encode_map(&tk, k_rot, s) ||
        !encode_map(&tgrads[1], a->dk, s) || !encode_map(&tgrads[2], a->dv, s) ||
        !encode_part_map(&tpart, part, s, S))
      return launch_error("frsa_bwd", cudaSuccess);
    e = frsa::launch_bwd_ordered(s, tq, tk, tv, tdo, to, tgrads[1], tgrads[2], tpart, a->o, a->d_o,
                                 a->lse, a->delta, a->cosp, a->sinp, a->dq, a->dk, a->dv, part, S,
                                 counters, delta_rows, &rot, st);
  }
  return e == cudaSuccess ? FRSA_OK : launch_error("frsa_bwd", e);
}

const char* frsa_last_error_detail(void) { return g_last_detail; }

int frsa_qkv_rope(const frsa_qkv_args* a, void* stream) {
  if (!a || !a->x || !a->w || !a->bias || !a->cosp || !a->sinp || !a->q || !a->k || !a->v)
    return FRSA_ERR_NULL_ARG;
  if (a->B < 1 || a->N < 1 || a->H < 1 || a->C < 1 || a->C % a->H != 0) return FRSA_ERR_BAD_SHAPE;
  if (a->has_cls != 0 && a->has_cls != 1) return FRSA_ERR_BAD_SHAPE;
  if (a->N - a->has_cls > a->n_pos) return FRSA_ERR_BAD_SHAPE;
  const long long D = a->C / a->H;
  if (a->C % 128 != 0 || D % 32 != 0 || D > 128) return FRSA_ERR_UNSUPPORTED_D;
  if (a->dtype != FRSA_DTYPE_BF16 && a->dtype != FRSA_DTYPE_F16) return FRSA_ERR_UNSUPPORTED_DTYPE;
  const long long M = a->B * a->N;
  if ((M + 127) / 128 * (3 * a->C / 128) > 0x7FFFFFFFLL || a->N > (1LL << 30))
    return FRSA_ERR_BAD_SHAPE;
  if (!aligned16(a->x) || !aligned16(a->w) || !aligned16(a->bias) || !aligned16(a->q) ||
      !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->cosp) || !aligned16(a->sinp))
    return FRSA_ERR_MISALIGNED;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  if (const int rc = pending_error("frsa_qkv_rope"); rc != FRSA_OK) return rc;
  const bool bf16 = a->dtype == FRSA_DTYPE_BF16;
  CUtensorMap tx, tw;
  if (!encode_map_2d(&tx, a->x, M, a->C, bf16) || !encode_map_2d(&tw, a->w, 3 * a->C, a->C, bf16))
    return launch_error("frsa_qkv_rope", cudaSuccess);
  const cudaError_t e = frsa::launch_qkv_rope(
      bf16, tx, tw, a->bias, a->cosp, a->sinp, a->q, a->k, a->v, M, static_cast<int>(a->N),
      static_cast<int>(a->C), static_cast<int>(a->H), static_cast<int>(D),
      static_cast<int>(a->has_cls), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FRSA_OK : launch_error("frsa_qkv_rope", e);
}

int frsa_qkv_rope_bwd(const frsa_qkv_bwd_args* a, void* stream) {
  if (!a || !a->dq || !a->dk || !a->dv || !a->cosp || !a->sinp || !a->dqkv)
    return FRSA_ERR_NULL_ARG;
  if (a->B < 1 || a->N < 1 || a->H < 1 || a->C < 1 || a->C % a->H != 0) return FRSA_ERR_BAD_SHAPE;
  if (a->has_cls != 0 && a->has_cls != 1) return FRSA_ERR_BAD_SHAPE;
  if (a->N - a->has_cls > a->n_pos) return FRSA_ERR_BAD_SHAPE;
  const long long D = a->C / a->H;
  if (a->C % 128 != 0 || D % 32 != 0 || D > 128) return FRSA_ERR_UNSUPPORTED_D;
  if (a->dtype != FRSA_DTYPE_BF16 && a->dtype != FRSA_DTYPE_F16) return FRSA_ERR_UNSUPPORTED_DTYPE;
  const long long M = a->B * a->N;
  if (M * (3 * a->C / 8) / 256 > 0x7FFFFFFFLL || a->N > (1LL << 30)) return FRSA_ERR_BAD_SHAPE;
  if (!aligned16(a->dq) || !aligned16(a->dk) || !aligned16(a->dv) || !aligned16(a->dqkv) ||
      !aligned16(a->cosp) || !aligned16(a->sinp))
    return FRSA_ERR_MISALIGNED;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  if (const int rc = pending_error("frsa_qkv_rope_bwd"); rc != FRSA_OK) return rc;
  const cudaError_t e = frsa::launch_qkv_rope_bwd(
      a->dtype == FRSA_DTYPE_BF16, a->dq, a->dk, a->dv, a->cosp, a->sinp, a->dqkv, M,
      static_cast<int>(a->N), static_cast<int>(a->C), static_cast<int>(a->H),
      static_cast<int>(D), static_cast<int>(a->has_cls), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FRSA_OK : launch_error("frsa_qkv_rope_bwd", e);
}

static int convert_common(const frsa_convert_args* a, bool in, const char* where, void* stream) {
  if (!a || !a->q || !a->k || !a->v || !a->q_out || !a->k_out || !a->v_out || !a->cosp ||
      !a->sinp)
    return FRSA_ERR_NULL_ARG;
  if (a->B < 1 || a->H < 1 || a->N < 1 || a->D < 8) return FRSA_ERR_BAD_SHAPE;
  if (a->has_cls != 0 && a->has_cls != 1) return FRSA_ERR_BAD_SHAPE;
  if (a->N - a->has_cls > a->n_pos) return FRSA_ERR_BAD_SHAPE;
  if (a->D % 8 != 0 || a->D > 128) return FRSA_ERR_UNSUPPORTED_D;
  if (a->dtype != FRSA_DTYPE_BF16 && a->dtype != FRSA_DTYPE_F16) return FRSA_ERR_UNSUPPORTED_DTYPE;
  const long long rows = a->B * a->H * a->N;
  if (rows * (a->D / 8) / 256 > 0x7FFFFFFFLL || a->N > (1LL << 30)) return FRSA_ERR_BAD_SHAPE;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->q_out) ||
      !aligned16(a->k_out) || !aligned16(a->v_out) || !aligned16(a->cosp) || !aligned16(a->sinp))
    return FRSA_ERR_MISALIGNED;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  if (const int rc = pending_error(where); rc != FRSA_OK) return rc;
  const void* src[3] = {a->q, a->k, a->v};
  void* dst[3] = {a->q_out, a->k_out, a->v_out};
  const cudaError_t e = frsa::launch_convert(
      in, a->dtype == FRSA_DTYPE_BF16, src, dst, a->cosp, a->sinp, rows, static_cast<int>(a->N),
      static_cast<int>(a->D), static_cast<int>(a->has_cls), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FRSA_OK : launch_error(where, e);
}

int frsa_convert_in(const frsa_convert_args* a, void* stream) {
  return convert_common(a, true, "frsa_convert_in", stream);
}

int frsa_convert_out(const frsa_convert_args* a, void* stream) {
  return convert_common(a, false, "frsa_convert_out", stream);
}

#ifdef FRSA_TRACE
// Trace builds only: copy the phase stamps (2048 CTAs x 64 slots) to `host`.
int frsa_trace_copy(unsigned long long* host, size_t n) {
  if (cudaDeviceSynchronize() != cudaSuccess) return FRSA_ERR_LAUNCH;
  return cudaMemcpyFromSymbol(host, frsa::g_trace, n * sizeof(unsigned long long)) ==
                 cudaSuccess ? FRSA_OK : FRSA_ERR_LAUNCH;
}
int frsa_trace_copy_it(unsigned long long* ts, unsigned int* fl, size_t n) {
  if (cudaDeviceSynchronize() != cudaSuccess) return FRSA_ERR_LAUNCH;
  if (cudaMemcpyFromSymbol(ts, frsa::g_trace_it, n * sizeof(unsigned long long)) != cudaSuccess)
    return FRSA_ERR_LAUNCH;
  return cudaMemcpyFromSymbol(fl, frsa::g_trace_fl, n * sizeof(unsigned int)) == cudaSuccess
             ? FRSA_OK : FRSA_ERR_LAUNCH;
}
#endif

int frsa_query_status(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return FRSA_ERR_LAUNCH;
  int st = 0;
  if (cudaMemcpyFromSymbol(&st, frsa::g_dev_status, sizeof(int)) != cudaSuccess)
    return FRSA_ERR_LAUNCH;
  if (st != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(frsa::g_dev_status, &zero, sizeof(int));
    return FRSA_ERR_DEVICE_TIMEOUT;
  }
  return FRSA_OK;
}

}  // extern "C"

// The allocation-free backward entry point (uses the helpers above).
#include "frsa_noalloc.cu"

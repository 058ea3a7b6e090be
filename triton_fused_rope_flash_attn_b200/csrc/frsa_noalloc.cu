// frsa_bwd_noalloc: the backward pass for callers that cannot allocate device
// memory.
//
// The general backward path needs an f32 dQ accumulation buffer of
// B*H*N*D floats, and frsa_bwd expects the caller to allocate it. Some callers
// cannot: a plugin host that hands a kernel only its input and output buffers
// and owns every allocation itself, a runtime whose memory pool is carved up
// before the first step, or a latency-critical loop that must not call
// cudaMalloc/cudaFree because they can synchronise the whole device. For them
// this entry point takes the accumulation buffer from a fixed array compiled
// into the library instead.
//
// Limits and sharing rules:
//   - The array holds kNoAllocScratchFloats floats (16 MiB). A call whose
//     B*H*N*D exceeds that is rejected with FRSA_ERR_SCRATCH_LIMIT before
//     anything is launched.
//   - Every GPU that loads the library keeps this array for the life of the
//     process.
//   - The array is shared by all calls on a device and keeps whatever the
//     last call left in it; each call clears the part it uses (an async memset
//     on the caller's stream) before accumulating. Two calls whose work
//     overlaps on the GPU (different streams, no ordering between them) race
//     on the array and produce wrong dQ. Order such calls on one stream.
//   - The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress while that device is current, and caches it. Make
//     that first call before any stream capture begins.
//
// This file is part of the single translation unit built from frsa_api.cu
// (it is included at the end of that file), so it reuses the validation and
// tensor-map helpers defined there and the backward kernels of frsa_bwd.cu.

#include <mutex>

namespace frsa {

// 4 Mi floats = 16 MiB of f32 dQ accumulation space per device.
constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;

// The scratch array. In host code this name is only a stand-in for the
// device symbol, never a usable address: host code must pass the address that
// cudaGetSymbolAddress returns (noalloc_scratch_ptr below).
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

namespace {

// Device address of g_noalloc_scratch on the current device, looked up once
// per device with that device current. Returns nullptr on failure.
float* noalloc_scratch_ptr() {
  static std::mutex mu;
  static float* cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<float*>(p);
  }
  return cache[dev];
}

// The general (key-tile per CTA, atomic dQ) backward with the given f32
// accumulation buffer, used for every shape.
template <typename T>
cudaError_t launch_bwd_accum_t(const LaunchShape& s, const CUtensorMap& tm_q,
                               const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               const CUtensorMap& tm_do, const CUtensorMap& tm_o,
                               const void* o, const float* lse,
                               float* delta, const float* cosp, const float* sinp, void* dq,
                               void* dk, void* dv, float* dq_accum, cudaStream_t stream) {
  const long long rows = static_cast<long long>(s.BH) * s.N;
  BwdParams p;
  p.cosp = cosp;
  p.sinp = sinp;
  p.lse = lse;
  p.o = o;
  p.delta_out = delta;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.dq_accum = dq_accum;
  p.BH = s.BH;
  p.N = s.N;
  p.D = s.D;
  p.nqt = (s.N + kTile - 1) / kTile;
  p.nkv = p.nqt;
  p.has_cls = s.has_cls;
  p.c2 = s.scale * 1.4426950408889634f;
  p.scale = s.scale;
  cudaError_t e =
      cudaMemsetAsync(dq_accum, 0, static_cast<size_t>(rows) * s.D * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  e = (s.D > 64) ? launch_bwd_main<T, 2, false>(s, tm_q, tm_k, tm_v, tm_do, tm_o, p, stream)
                 : launch_bwd_main<T, 1, false>(s, tm_q, tm_k, tm_v, tm_do, tm_o, p, stream);
  if (e != cudaSuccess) return e;
  const int threads = 256;
  const long long total = rows * (s.D >> 3);
  dq_finalize_kernel<T><<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0,
                          stream>>>(dq_accum, static_cast<T*>(dq), cosp, sinp, rows, s.N, s.D,
                                    s.has_cls);
  return cudaGetLastError();
}

}  // namespace
}  // namespace frsa

extern "C" size_t frsa_bwd_noalloc_max_elements(void) { return frsa::kNoAllocScratchFloats; }

extern "C" int frsa_bwd_noalloc(const frsa_attn_args* a, void* stream) {
  frsa::LaunchShape s;
  int rc = validate_common(a, &s);
  if (rc != FRSA_OK) return rc;
  if (s.f32) return FRSA_ERR_UNSUPPORTED_DTYPE;   // 16-bit kernels only
  if (!a->o || !a->lse || !a->d_o || !a->dq || !a->dk || !a->dv) return FRSA_ERR_NULL_ARG;
  if (!aligned16(a->o) || !aligned16(a->d_o) || !aligned16(a->dq) || !aligned16(a->dk) ||
      !aligned16(a->dv) || !aligned16(a->lse))
    return FRSA_ERR_MISALIGNED;
  const size_t need = static_cast<size_t>(s.BH) * s.N * s.D;
  if (need > frsa::kNoAllocScratchFloats) return FRSA_ERR_SCRATCH_LIMIT;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  float* scratch = frsa::noalloc_scratch_ptr();
  if (scratch == nullptr) return launch_error("frsa_bwd_noalloc: cudaGetSymbolAddress", cudaGetLastError());
  (void)cudaGetLastError();
  CUtensorMap tq, tk, tv, tdo, to;
  if (!encode_map(&tq, a->q, s) || !encode_map(&tk, a->k, s) || !encode_map(&tv, a->v, s) ||
      !encode_map(&tdo, a->d_o, s) || !encode_map(&to, a->o, s))
    return launch_error("frsa_bwd_noalloc", cudaSuccess);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      s.bf16 ? frsa::launch_bwd_accum_t<__nv_bfloat16>(s, tq, tk, tv, tdo, to, a->o, a->lse, a->delta,
                                                       a->cosp, a->sinp, a->dq, a->dk, a->dv,
                                                       scratch, st)
             : frsa::launch_bwd_accum_t<__half>(s, tq, tk, tv, tdo, to, a->o, a->lse, a->delta,
                                                a->cosp, a->sinp, a->dq, a->dk, a->dv, scratch,
                                                st);
  return e == cudaSuccess ? FRSA_OK : launch_error("frsa_bwd_noalloc", e);
}

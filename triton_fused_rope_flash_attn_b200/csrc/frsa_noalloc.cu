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
//   - The array holds kNoAllocScratchFloats floats (16 MiB) of dQ running
//     sums plus kNoAllocCounterInts int32 words (4 MiB) of counters. A
//     call whose B*H*N*D exceeds kNoAllocScratchFloats is rejected with
//     FRSA_ERR_SCRATCH_LIMIT before anything is launched.
//   - Every GPU that loads the library keeps this array for the life of the
//     process.
//   - The array is shared by all calls on a device and keeps whatever the
//     last call left in it. Each call clears the counters it uses (an async
//     memset on the caller's stream); the running sums need no clearing (the
//     first key tile of every query tile stores instead of adding). Two calls
//     whose work overlaps on the GPU (different streams, no ordering between
//     them) race on the array and produce wrong dQ. Order such calls on one
//     stream.
//   - The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress while that device is current, and caches it. Make
//     that first call before any stream capture begins. The cached address
//     assumes the device's primary context lives as long as the process: after
//     cudaDeviceReset the library must not be used again in that process.
//
// This file is part of the single translation unit built from frsa_api.cu
// (it is included at the end of that file), so it reuses the validation and
// tensor-map helpers defined there and the backward kernels of frsa_bwd.cu.

#include <mutex>

namespace frsa {

// 4 Mi floats = 16 MiB of f32 dQ running sums per device.
constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;
// Counters: an arrival and a slot-turn counter per (head, 128-query tile) with
// one slot, plus the claim ticket. With B*H*N*D <= 4 Mi and D >= 8 there are
// at most 512 Ki (head, query tile) pairs.
constexpr size_t kNoAllocCounterInts = (size_t(1024) << 10) + 4;

// The scratch array (running sums, then counters). In host code this name is
// only a stand-in for the device symbol, never a usable address: host code
// must pass the address that cudaGetSymbolAddress returns (noalloc_scratch_ptr
// below).
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats + kNoAllocCounterInts];

namespace {

// Device address of g_noalloc_scratch on the current device, looked up once
// per device with that device current. Returns nullptr on failure (the CUDA
// error of the lookup is then consumed and reported by the caller).
float* noalloc_scratch_ptr(cudaError_t* err) {
  static std::mutex mu;
  static float* cache[64] = {};
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (*err != cudaSuccess) {
      (void)cudaGetLastError();   // the lookup's own error, reported to the caller
      return nullptr;
    }
    cache[dev] = static_cast<float*>(p);
  }
  return cache[dev];
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
      !aligned16(a->dv) || !aligned16(a->lse) || (a->delta && !aligned16(a->delta)))
    return FRSA_ERR_MISALIGNED;
  const size_t need = static_cast<size_t>(s.BH) * s.N * s.D;
  if (need > frsa::kNoAllocScratchFloats) return FRSA_ERR_SCRATCH_LIMIT;
  // As many partial slots as the array holds (at most frsa_bwd's count);
  // with fewer slots, key tiles that share one take turns.
  int S = frsa::bwd_slots(s);
  while (S > 1 && (S * need > frsa::kNoAllocScratchFloats ||
                   frsa::bwd_counter_ints(s, S) > frsa::kNoAllocCounterInts))
    --S;
  if (frsa::bwd_counter_ints(s, S) > frsa::kNoAllocCounterInts) return FRSA_ERR_SCRATCH_LIMIT;
  if (!device_is_sm100()) return FRSA_ERR_NO_DEVICE;
  if ((rc = pending_error("frsa_bwd_noalloc")) != FRSA_OK) return rc;
  cudaError_t lookup = cudaSuccess;
  float* scratch = frsa::noalloc_scratch_ptr(&lookup);
  if (scratch == nullptr) return launch_error("frsa_bwd_noalloc: cudaGetSymbolAddress", lookup);
  CUtensorMap tq, tk, tv, tdo, to;
  if (!encode_map(&tq, a->q, s, false, strides_of(a->q_strides)) ||
      !encode_map(&tk, a->k, s, false, strides_of(a->k_strides)) ||
      !encode_map(&tv, a->v, s, false, strides_of(a->v_strides)) ||
      !encode_map(&tdo, a->d_o, s) || !encode_map(&to, a->o, s))
    return launch_error("frsa_bwd_noalloc", cudaSuccess);
  // Every shape (also N <= 256, D <= 64) runs the general key-tile kernel
  // here; Delta comes from a pre-pass into the caller's `delta` when given,
  // else it is formed inside the kernel.
  int* counters = reinterpret_cast<int*>(scratch + frsa::kNoAllocScratchFloats);
  CUtensorMap tdk, tdv, tpart;
  if (!encode_map(&tdk, a->dk, s) || !encode_map(&tdv, a->dv, s) ||
      !encode_part_map(&tpart, scratch, s, S))
    return launch_error("frsa_bwd_noalloc", cudaSuccess);
  const cudaError_t e = frsa::launch_bwd_ordered(
      s, tq, tk, tv, tdo, to, tdk, tdv, tpart, a->o, a->d_o, a->lse, a->delta, a->cosp, a->sinp,
      a->dq, a->dk, a->dv, scratch, S, counters, a->delta, /*rot=*/nullptr,
      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FRSA_OK : launch_error("frsa_bwd_noalloc", e);
}

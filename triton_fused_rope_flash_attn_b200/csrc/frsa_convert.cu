// f32 inputs under 16-bit autocast (the reference converts its f32 loads to
// the compute type, fa_rope_full .py:168-174, 240-246):
//
//   convert_in   q, k, v f32 [B, H, N, D] -> q^ = R(q), k^ = R(k), v in the
//                16-bit compute type, rotated in f32 and rounded once, so the
//                attention kernels then run without rotation
//                (FRSA_FLAG_NO_ROPE);
//   convert_out  dq^, dk^, dv (16-bit, with respect to q^, k^, v) ->
//                dq = R^T dq^, dk = R^T dk^, dv in f32.
//
// One thread per 8-element granule; every tensor is read and written once.
#include "frsa_internal.h"
#include "frsa_ptx.cuh"
#include "frsa_rope.cuh"

namespace frsa {

namespace {

struct ConvertParams {
  const void* src[3];
  void* dst[3];
  const float* cosp;
  const float* sinp;
  long long granules;   // per tensor: B * H * N * D / 8
  int N, D, has_cls;
};

template <typename T>
__global__ void convert_in_kernel(const ConvertParams p) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int which = blockIdx.y;   // 0 q, 1 k, 2 v
  if (idx >= p.granules) return;
  const int G = p.D >> 3;
  const long long row = idx / G;
  const int gg = static_cast<int>(idx - row * G);
  const float4* s = reinterpret_cast<const float4*>(p.src[which]) + 2 * idx;
  const float4 a = __ldcs(s), b = __ldcs(s + 1);
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const int pos = which < 2 ? rope_pos(static_cast<int>(row % p.N), p.N, p.has_cls) : -1;
  if (pos >= 0) {
    const size_t t0 = static_cast<size_t>(pos) * (p.D >> 1) + 4 * gg;
    const float4 c = __ldg(reinterpret_cast<const float4*>(p.cosp + t0));
    const float4 sn = __ldg(reinterpret_cast<const float4*>(p.sinp + t0));
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {   // the reference's pair rotation (even, odd)
      const float e = v[2 * q], o = v[2 * q + 1];
      v[2 * q] = e * cc[q] - o * ss[q];
      v[2 * q + 1] = o * cc[q] + e * ss[q];
    }
  }
  reinterpret_cast<uint4*>(p.dst[which])[idx] = pack8<T>(v);
}

template <typename T>
__global__ void convert_out_kernel(const ConvertParams p) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int which = blockIdx.y;   // 0 dq, 1 dk, 2 dv
  if (idx >= p.granules) return;
  const int G = p.D >> 3;
  const long long row = idx / G;
  const int gg = static_cast<int>(idx - row * G);
  const uint4 x = __ldcs(reinterpret_cast<const uint4*>(p.src[which]) + idx);
  float v[8];
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = Elt<T>::unpack(w[e]);
    v[2 * e] = t.x;
    v[2 * e + 1] = t.y;
  }
  const int pos = which < 2 ? rope_pos(static_cast<int>(row % p.N), p.N, p.has_cls) : -1;
  if (pos >= 0) {
    const size_t t0 = static_cast<size_t>(pos) * (p.D >> 1) + 4 * gg;
    unrotate8(v, __ldg(reinterpret_cast<const float4*>(p.cosp + t0)),
              __ldg(reinterpret_cast<const float4*>(p.sinp + t0)));
  }
  float4* d = reinterpret_cast<float4*>(p.dst[which]) + 2 * idx;
  d[0] = make_float4(v[0], v[1], v[2], v[3]);
  d[1] = make_float4(v[4], v[5], v[6], v[7]);
}

}  // namespace

cudaError_t launch_convert(bool in, bool bf16, const void* const* src, void* const* dst,
                           const float* cosp, const float* sinp, long long rows, int N, int D,
                           int has_cls, cudaStream_t stream) {
  ConvertParams p;
  for (int i = 0; i < 3; ++i) {
    p.src[i] = src[i];
    p.dst[i] = dst[i];
  }
  p.cosp = cosp;
  p.sinp = sinp;
  p.granules = rows * (D / 8);
  p.N = N;
  p.D = D;
  p.has_cls = has_cls;
  if (p.granules == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((p.granules + 255) / 256), 3);
  if (in) {
    if (bf16) convert_in_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p);
    else convert_in_kernel<__half><<<grid, 256, 0, stream>>>(p);
  } else {
    if (bf16) convert_out_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p);
    else convert_out_kernel<__half><<<grid, 256, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace frsa

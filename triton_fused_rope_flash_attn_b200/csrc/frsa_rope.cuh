// In-shared-memory 2D-RoPE rotation of one tile row, plus the R^T un-rotation
// used by the backward epilogues.
//
// A tile is NCH chunks of [128 rows][64 cols] 16-bit elements, each chunk in the
// 128-byte-swizzled layout TMA writes (granule g of row r at (g ^ (r & 7)) * 16).
// Pair p of a row is the 32-bit word holding columns (2p, 2p+1); a 16-byte
// granule holds pairs 4g'..4g'+3, so the swizzle never splits a pair.
//
// Rotation of pair (e, o) with table values (c, s) (fa_rope_full .py:201-202,
// 271-272):  e' = e c - o s,  o' = o c + e s.  Token t uses table row t - has_cls;
// the CLS token (t == 0 with has_cls) is left as is (fa_rope_full .py:177-179).
// The arithmetic is f32 with one rounding to the 16-bit type.
#pragma once
#include "frsa_ptx.cuh"

namespace frsa {

// Table row index of token `t`, or -1 when the token is not rotated.
__device__ __forceinline__ int rope_pos(int t, int N, int has_cls) {
  if (t >= N) return -1;
  if (has_cls && t == 0) return -1;
  return t - has_cls;
}

template <typename T, int NCH>
__device__ __forceinline__ void rotate_row_smem(uint8_t* tile, int r, int D, int pos,
                                                const float* __restrict__ cosp,
                                                const float* __restrict__ sinp) {
  if (pos < 0) return;
  const int D2 = D >> 1;
  const float4* crow = reinterpret_cast<const float4*>(cosp + static_cast<size_t>(pos) * D2);
  const float4* srow = reinterpret_cast<const float4*>(sinp + static_cast<size_t>(pos) * D2);
  const int ngran = D >> 3;  // 8 elements = 4 pairs per granule
#pragma unroll
  for (int gg = 0; gg < 8 * NCH; ++gg) {
    if (gg < ngran) {
      const int c = gg >> 3, g = gg & 7;
      uint4* p = reinterpret_cast<uint4*>(tile + c * 16384 + sw128_off(r, g));
      uint4 w = *p;
      const float4 cs = __ldg(crow + gg);
      const float4 sn = __ldg(srow + gg);
      float2 a = Elt<T>::unpack(w.x), b = Elt<T>::unpack(w.y), cc = Elt<T>::unpack(w.z),
             d = Elt<T>::unpack(w.w);
      w.x = Elt<T>::pack(a.x * cs.x - a.y * sn.x, a.y * cs.x + a.x * sn.x);
      w.y = Elt<T>::pack(b.x * cs.y - b.y * sn.y, b.y * cs.y + b.x * sn.y);
      w.z = Elt<T>::pack(cc.x * cs.z - cc.y * sn.z, cc.y * cs.z + cc.x * sn.z);
      w.w = Elt<T>::pack(d.x * cs.w - d.y * sn.w, d.y * cs.w + d.x * sn.w);
      *p = w;
    }
  }
}

// R^T on an f32 row held in registers (v[2p], v[2p+1] = gradient of pair p in
// the rotated basis):  e = e^ c + o^ s,  o = -e^ s + o^ c  (fa_rope_full .py:653-662).
template <int NV>
__device__ __forceinline__ void unrotate_row_regs(float (&v)[NV], int D, int pos,
                                                  const float* __restrict__ cosp,
                                                  const float* __restrict__ sinp) {
  if (pos < 0) return;
  const int D2 = D >> 1;
  const float* crow = cosp + static_cast<size_t>(pos) * D2;
  const float* srow = sinp + static_cast<size_t>(pos) * D2;
#pragma unroll
  for (int p = 0; p < NV / 2; ++p) {
    if (p < D2) {
      const float c = __ldg(crow + p), s = __ldg(srow + p);
      const float e = v[2 * p], o = v[2 * p + 1];
      v[2 * p] = e * c + o * s;
      v[2 * p + 1] = o * c - e * s;
    }
  }
}

// Store an f32 row of D values as 16-bit elements (D % 8 == 0, dst 16-byte aligned).
template <typename T, int NV>
__device__ __forceinline__ void store_row(T* dst, const float (&v)[NV], int D) {
#pragma unroll
  for (int g = 0; g < NV / 8; ++g) {
    if (g * 8 < D) {
      uint4 w;
      w.x = Elt<T>::pack(v[8 * g + 0], v[8 * g + 1]);
      w.y = Elt<T>::pack(v[8 * g + 2], v[8 * g + 3]);
      w.z = Elt<T>::pack(v[8 * g + 4], v[8 * g + 5]);
      w.w = Elt<T>::pack(v[8 * g + 6], v[8 * g + 7]);
      reinterpret_cast<uint4*>(dst)[g] = w;
    }
  }
}

}  // namespace frsa

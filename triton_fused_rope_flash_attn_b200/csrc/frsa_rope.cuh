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

// Pull the table rows of token position `pos` toward L1 ahead of use, so the
// rotation that follows a TMA wait does not pay an L2 round trip per granule.
__device__ __forceinline__ void prefetch_rope_row(int pos, int D, const float* __restrict__ cosp,
                                                  const float* __restrict__ sinp) {
  if (pos < 0) return;
  const int D2 = D >> 1;
  const char* c = reinterpret_cast<const char*>(cosp + static_cast<size_t>(pos) * D2);
  const char* s = reinterpret_cast<const char*>(sinp + static_cast<size_t>(pos) * D2);
  for (int off = 0; off < D2 * 4; off += 128) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(c + off));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(s + off));
  }
}

// Rotate row r of a tile in place. Granules are processed four at a time with
// every shared and table load of the group issued before any store, so the
// loads overlap (the stores go through a generic pointer the compiler must
// assume may alias the tables).
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
  for (int g0 = 0; g0 < 8 * NCH; g0 += 4) {
    if (g0 < ngran) {
      uint4 w[4];
      float4 cs[4], sn[4];
      uint4* ptr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int gg = g0 + u;
        ptr[u] = reinterpret_cast<uint4*>(tile + (gg >> 3) * 16384 + sw128_off(r, gg & 7));
        if (gg < ngran) {
          w[u] = *ptr[u];
          cs[u] = __ldg(crow + gg);
          sn[u] = __ldg(srow + gg);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (g0 + u < ngran) {
          const float2 a = Elt<T>::unpack(w[u].x), b = Elt<T>::unpack(w[u].y),
                       cc = Elt<T>::unpack(w[u].z), d = Elt<T>::unpack(w[u].w);
          const float4 c = cs[u], s = sn[u];
          uint4 o;
          o.x = Elt<T>::pack(a.x * c.x - a.y * s.x, a.y * c.x + a.x * s.x);
          o.y = Elt<T>::pack(b.x * c.y - b.y * s.y, b.y * c.y + b.x * s.y);
          o.z = Elt<T>::pack(cc.x * c.z - cc.y * s.z, cc.y * c.z + cc.x * s.z);
          o.w = Elt<T>::pack(d.x * c.w - d.y * s.w, d.y * c.w + d.x * s.w);
          *ptr[u] = o;
        }
      }
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

namespace frsa {

// ---------------------------------------------------------------------------
// Warp-per-row helpers. A warp walks rows [r_begin, r_end) of a tile; lane p
// owns RoPE pair p (columns 2p, 2p+1), so table reads are coalesced (one
// 128-byte line per row for D = 64) and shared-memory accesses of a row hit 32
// distinct banks.

// Byte offset of pair p of row r in a 128B-swizzled chunked tile.
__device__ __forceinline__ uint32_t sw128_pair_off(uint32_t r, uint32_t p) {
  const uint32_t c = p >> 5, q = p & 31;
  return c * 16384u + r * 128u + ((((q >> 2) ^ (r & 7u))) << 4) + ((q & 3u) << 2);
}

// Table values for the 32 rows a warp rotates, lane p holding pair p
// (D <= 64) or pairs p and p + 32 (D <= 128). Loaded before the tile's TMA
// wait so the table latency overlaps the load.
template <int NCH, int ROWS = 32>
struct RopeRows {
  float c[NCH][ROWS], s[NCH][ROWS];
};

template <int NCH, int ROWS = 32>
__device__ __forceinline__ void load_rope_rows(RopeRows<NCH, ROWS>& t, int r_begin, int tok0, int N,
                                               int has_cls, int D,
                                               const float* __restrict__ cosp,
                                               const float* __restrict__ sinp, int lane) {
  const int D2 = D >> 1;
#pragma unroll
  for (int h = 0; h < NCH; ++h) {
    const int p = lane + 32 * h;
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
      const int pos = rope_pos(tok0 + r_begin + u, N, has_cls);
      t.c[h][u] = 1.f;
      t.s[h][u] = 0.f;
      if (pos >= 0 && p < D2) {
        t.c[h][u] = __ldg(cosp + static_cast<size_t>(pos) * D2 + p);
        t.s[h][u] = __ldg(sinp + static_cast<size_t>(pos) * D2 + p);
      }
    }
  }
}

// Rotate the warp's ROWS rows [r_begin, r_begin + ROWS) of a tile in place
// with preloaded table values (rows that are not rotated carry c = 1, s = 0).
template <typename T, int NCH, int ROWS = 32>
__device__ __forceinline__ void apply_rope_rows(uint8_t* tile, int r_begin, int D,
                                                const RopeRows<NCH, ROWS>& t, int lane) {
  const int D2 = D >> 1;
  const uint32_t base = smem_u32(tile);
#pragma unroll
  for (int h = 0; h < NCH; ++h) {
    const int p = lane + 32 * h;
    if (p < D2) {
      uint32_t w[ROWS];
#pragma unroll
      for (int u = 0; u < ROWS; ++u) w[u] = lds_u32(base + sw128_pair_off(r_begin + u, p));
#pragma unroll
      for (int u = 0; u < ROWS; ++u) {
        const float2 x = Elt<T>::unpack(w[u]);
        const float c = t.c[h][u], s = t.s[h][u];
        sts_u32(base + sw128_pair_off(r_begin + u, p),
                Elt<T>::pack(x.x * c - x.y * s, x.y * c + x.x * s));
      }
    }
  }
}

// Row stride and swizzle of the f32 staging tile used by the epilogues:
// rows of 64*NCH floats, 16-byte chunk c of row r stored at chunk c ^ (r & 7).
template <int NCH>
__device__ __forceinline__ uint32_t stage_off(uint32_t r, uint32_t chunk) {
  return r * (256u * NCH) + ((chunk ^ (r & 7u)) << 4);
}

// Thread-per-row write of 16 consecutive f32 values (columns 16*c16 ..) of row r.
template <int NCH>
__device__ __forceinline__ void stage_write16(uint8_t* stage, int r, int c16, const float (&v)[16]) {
  const uint32_t base = smem_u32(stage);
#pragma unroll
  for (int u = 0; u < 4; ++u)
    sts_f4(base + stage_off<NCH>(r, c16 * 4 + u),
           make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]));
}

// Warp-per-row drain of the warp's ROWS staged f32 rows [r_begin, r_begin + ROWS):
// scale, optional R^T un-rotation with preloaded tables (pass rope = nullptr
// for none), rounding to T and a coalesced store to dst + tok * D for the rows
// whose token tok0 + r is < N.
template <typename T, int NCH, int ROWS = 32>
__device__ __forceinline__ void drain_rows_warp(const uint8_t* stage, int r_begin, int tok0, int N,
                                                int D, float scale,
                                                const RopeRows<NCH, ROWS>* rope, T* dst,
                                                int lane) {
  const int D2 = D >> 1;
  const uint32_t base = smem_u32(stage);
#pragma unroll
  for (int h = 0; h < NCH; ++h) {
    const int p = lane + 32 * h;
    if (p < D2) {
#pragma unroll
      for (int u = 0; u < ROWS; ++u) {
        const int r = r_begin + u;
        const int tok = tok0 + r;
        if (tok < N) {
          const float2 g = lds_f2(base + stage_off<NCH>(r, p >> 1) + ((p & 1) << 3));
          float e = g.x * scale, o = g.y * scale;
          if (rope != nullptr) {
            const float c = rope->c[h][u], s = rope->s[h][u];
            const float e2 = e * c + o * s;
            o = o * c - e * s;
            e = e2;
          }
          reinterpret_cast<uint32_t*>(dst + static_cast<size_t>(tok) * D)[p] = Elt<T>::pack(e, o);
        }
      }
    }
  }
}

}  // namespace frsa

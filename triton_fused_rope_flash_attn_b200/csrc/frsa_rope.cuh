// 2D-RoPE rotation of shared-memory tiles, R^T un-rotation in the epilogues,
// and the row-wise helpers the kernels share.
//
// A tile is NCH chunks of [128 rows][64 cols] 16-bit elements, each chunk in the
// 128-byte-swizzled layout TMA writes (16-byte granule g of row r at
// (g ^ (r & 7)) * 16). Pair p of a row is the 32-bit word holding columns
// (2p, 2p+1); granule g holds pairs 4g .. 4g+3, so the swizzle never splits a
// pair.
//
// Rotation of pair (e, o) with table values (c, s) (fa_rope_full .py:201-202,
// 271-272):  e' = e c - o s,  o' = o c + e s.  Token t uses table row
// t - has_cls; the CLS token (t == 0 with has_cls) is left as is
// (fa_rope_full .py:177-179). Gradients are un-rotated with R^T
// (fa_rope_full .py:653-662, 984-993):  e = e^ c + o^ s,  o = o^ c - e^ s.
// All arithmetic is f32 with one rounding to the 16-bit type.
//
// Row-wise work uses a "quad" layout: a warp handles 4 rows per instruction,
// lane l taking granule (l & 7) of row (l >> 3) of the quad, so every
// shared-memory access is a conflict-free 16-byte vector and every global
// access of a row is one coalesced 128-byte line. (With one lane per pair the
// count of shared-memory instructions, not their latency, bounds these loops.)
#pragma once
#include "frsa_ptx.cuh"

namespace frsa {

// Table row index of token `t`, or -1 when the token is not rotated.
// has_cls < 0 marks a call without RoPE (q and k arrive rotated): no token is.
__device__ __forceinline__ int rope_pos(int t, int N, int has_cls) {
  if (t >= N || has_cls < 0) return -1;
  if (has_cls && t == 0) return -1;
  return t - has_cls;
}

// Rotate the four pairs of a granule.
template <typename T>
__device__ __forceinline__ uint4 rotate_granule(uint4 x, float4 c, float4 s) {
  uint4 o;
  float2 v;
  v = Elt<T>::unpack(x.x);
  o.x = Elt<T>::pack(v.x * c.x - v.y * s.x, v.y * c.x + v.x * s.x);
  v = Elt<T>::unpack(x.y);
  o.y = Elt<T>::pack(v.x * c.y - v.y * s.y, v.y * c.y + v.x * s.y);
  v = Elt<T>::unpack(x.z);
  o.z = Elt<T>::pack(v.x * c.z - v.y * s.z, v.y * c.z + v.x * s.z);
  v = Elt<T>::unpack(x.w);
  o.w = Elt<T>::pack(v.x * c.w - v.y * s.w, v.y * c.w + v.x * s.w);
  return o;
}

// Table values for ROWS rows of a tile (ROWS / 4 quads), lane l holding the
// four pairs of granule (l & 7) (+ 8 h for chunk h) of its row of each quad.
// Rows that are not rotated hold c = 1, s = 0. Loaded before a tile's TMA wait
// so the global-memory latency overlaps the load.
template <int NCH, int ROWS>
struct RopeQ {
  float4 c[NCH][ROWS / 4], s[NCH][ROWS / 4];
};

template <int NCH, int ROWS>
__device__ __forceinline__ void load_rope_q(RopeQ<NCH, ROWS>& t, int r_begin, int tok0, int N,
                                            int has_cls, int D, const float* __restrict__ cosp,
                                            const float* __restrict__ sinp, int lane) {
  const int D2 = D >> 1;
  const int rq = lane >> 3, gl = lane & 7;
#pragma unroll
  for (int k = 0; k < ROWS / 4; ++k) {
    const int pos = rope_pos(tok0 + r_begin + 4 * k + rq, N, has_cls);
#pragma unroll
    for (int h = 0; h < NCH; ++h) {
      const int g = gl + 8 * h;
      t.c[h][k] = make_float4(1.f, 1.f, 1.f, 1.f);
      t.s[h][k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (pos >= 0 && 8 * g < D) {
        t.c[h][k] = __ldg(reinterpret_cast<const float4*>(cosp + static_cast<size_t>(pos) * D2) + g);
        t.s[h][k] = __ldg(reinterpret_cast<const float4*>(sinp + static_cast<size_t>(pos) * D2) + g);
      }
    }
  }
}

// Rotate rows [r_begin, r_begin + ROWS) of a tile in place with preloaded tables.
template <typename T, int NCH, int ROWS>
__device__ __forceinline__ void apply_rope_q(uint8_t* tile, int r_begin, int D,
                                             const RopeQ<NCH, ROWS>& t, int lane) {
  const uint32_t base = smem_u32(tile);
  const int rq = lane >> 3, gl = lane & 7;
  uint4 x[NCH][ROWS / 4];
#pragma unroll
  for (int k = 0; k < ROWS / 4; ++k)
#pragma unroll
    for (int h = 0; h < NCH; ++h)
      if (8 * (gl + 8 * h) < D)
        x[h][k] = lds_u4(base + h * 16384 + sw128_off(r_begin + 4 * k + rq, gl));
#pragma unroll
  for (int k = 0; k < ROWS / 4; ++k)
#pragma unroll
    for (int h = 0; h < NCH; ++h)
      if (8 * (gl + 8 * h) < D)
        sts_u4(base + h * 16384 + sw128_off(r_begin + 4 * k + rq, gl),
               rotate_granule<T>(x[h][k], t.c[h][k], t.s[h][k]));
}

// Rotate `nrows` rows (a multiple of 16) from r_begin of a one-chunk tile in
// place, with the tables resident in shared memory as [n_pos][32] f32 (D <= 64).
template <typename T>
__device__ __forceinline__ void rotate_q_tabsm(uint32_t tile, int r_begin, int nrows, int tok0,
                                               int N, int has_cls, int D, uint32_t cos_sm,
                                               uint32_t sin_sm, int lane) {
  const int rq = lane >> 3, gl = lane & 7;
  if (8 * gl >= D) return;
  for (int u0 = 0; u0 < nrows; u0 += 16) {
    uint4 x[4];
    float4 c[4], s[4];
    int pos[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = r_begin + u0 + 4 * k + rq;
      pos[k] = rope_pos(tok0 + r, N, has_cls);
      const int pq = pos[k] < 0 ? 0 : pos[k];
      c[k] = lds_f4(cos_sm + (pq * 32 + 4 * gl) * 4);
      s[k] = lds_f4(sin_sm + (pq * 32 + 4 * gl) * 4);
      x[k] = lds_u4(tile + sw128_off(r, gl));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (pos[k] >= 0)
        sts_u4(tile + sw128_off(r_begin + u0 + 4 * k + rq, gl),
               rotate_granule<T>(x[k], c[k], s[k]));
  }
}

// ---------------------------------------------------------------------------
// f32 staging tile used by the epilogues: rows of 64*NCH floats, 16-byte chunk
// c of row r stored at chunk c ^ (r & 7). Rows are written thread-per-row (the
// TMEM read-out layout) and drained in the quad layout.
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

// Read granule g (8 floats) of staged row r, scaled.
template <int NCH>
__device__ __forceinline__ void stage_read8(uint32_t base, int r, int g, float scale,
                                            float (&v)[8]) {
  const float4 a = lds_f4(base + stage_off<NCH>(r, 2 * g));
  const float4 b = lds_f4(base + stage_off<NCH>(r, 2 * g + 1));
  v[0] = a.x * scale; v[1] = a.y * scale; v[2] = a.z * scale; v[3] = a.w * scale;
  v[4] = b.x * scale; v[5] = b.y * scale; v[6] = b.z * scale; v[7] = b.w * scale;
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 w;
  w.x = Elt<T>::pack(v[0], v[1]);
  w.y = Elt<T>::pack(v[2], v[3]);
  w.z = Elt<T>::pack(v[4], v[5]);
  w.w = Elt<T>::pack(v[6], v[7]);
  return w;
}

// R^T on the four pairs of a granule held as 8 floats.
__device__ __forceinline__ void unrotate8(float (&v)[8], float4 c, float4 s) {
  const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float e = v[2 * p], o = v[2 * p + 1];
    v[2 * p] = e * cc[p] + o * ss[p];
    v[2 * p + 1] = o * cc[p] - e * ss[p];
  }
}

// Drain staged rows [r_begin, r_begin + ROWS): scale, optional R^T with
// preloaded tables (rope == nullptr for none), round to T, store to
// dst + tok * D with tok = tok0 + r (rows with tok >= N are skipped).
template <typename T, int NCH, int ROWS>
__device__ __forceinline__ void drain_q(const uint8_t* stage, int r_begin, int tok0, int N, int D,
                                        float scale, const RopeQ<NCH, ROWS>* rope, T* dst,
                                        int lane) {
  const uint32_t base = smem_u32(stage);
  const int rq = lane >> 3, gl = lane & 7;
#pragma unroll
  for (int k = 0; k < ROWS / 4; ++k) {
    const int r = r_begin + 4 * k + rq;
    const int tok = tok0 + r;
#pragma unroll
    for (int h = 0; h < NCH; ++h) {
      const int g = gl + 8 * h;
      if (tok < N && 8 * g < D) {
        float v[8];
        stage_read8<NCH>(base, r, g, scale, v);
        if (rope != nullptr) unrotate8(v, rope->c[h][k], rope->s[h][k]);
        *reinterpret_cast<uint4*>(dst + static_cast<size_t>(tok) * D + 8 * g) = pack8<T>(v);
      }
    }
  }
}

// Drain one 64-column block of O: the stage (one-chunk layout) holds columns
// [64 blk, 64 blk + 64) of rows [r_begin, r_begin + ROWS).
template <typename T, int ROWS>
__device__ __forceinline__ void drain_block_q(const uint8_t* stage, int r_begin, int tok0, int N,
                                              int D, int blk, T* dst, int lane) {
  const uint32_t base = smem_u32(stage);
  const int rq = lane >> 3, gl = lane & 7;
  const int g = 8 * blk + gl;
  if (8 * g >= D) return;
#pragma unroll
  for (int k = 0; k < ROWS / 4; ++k) {
    const int r = r_begin + 4 * k + rq;
    const int tok = tok0 + r;
    if (tok < N) {
      float v[8];
      stage_read8<1>(base, r, gl, 1.f, v);
      *reinterpret_cast<uint4*>(dst + static_cast<size_t>(tok) * D + 8 * g) = pack8<T>(v);
    }
  }
}

}  // namespace frsa

namespace frsa {

// ---------------------------------------------------------------------------
// Thread-per-row helpers (thread = tile row = TMEM lane), used where a row's
// values arrive in one thread's registers from TMEM. Table values live in a
// shared "table tile" laid out like a data tile: granule g of row r holds the
// four pairs 4g..4g+3 of that row as packed f16 (cos, sin) (low half cos).
// cos and sin lie in [-1, 1], so f16 keeps them to ~2^-11 relative, far below
// the 16-bit rounding of the rotated values themselves.

// Write row r of a table tile for token position pos (pos < 0: identity).
__device__ __forceinline__ void store_tabrow(uint32_t tab, int r, int pos, int D,
                                             const float* __restrict__ cosp,
                                             const float* __restrict__ sinp) {
  const int D2 = D >> 1;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    float4 c = make_float4(1.f, 1.f, 1.f, 1.f), s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (pos >= 0 && 8 * g < D) {
      c = __ldg(reinterpret_cast<const float4*>(cosp + static_cast<size_t>(pos) * D2) + g);
      s = __ldg(reinterpret_cast<const float4*>(sinp + static_cast<size_t>(pos) * D2) + g);
    }
    sts_u4(tab + sw128_off(r, g),
           make_uint4(Elt<__half>::pack(c.x, s.x), Elt<__half>::pack(c.y, s.y),
                      Elt<__half>::pack(c.z, s.z), Elt<__half>::pack(c.w, s.w)));
  }
}

// Rotate row r of a one-chunk tile in place with table tile `tab`, kBatch
// granules at a time: with kBatch > 1 all of a batch's shared loads are issued
// before its first store (the loads and stores are ordered asm), so their
// latencies overlap, at the cost of 8 registers per granule in flight.
template <typename T, int kBatch = 1>
__device__ __forceinline__ void rotate_row_t(uint32_t tile, uint32_t tab, int r, int D) {
#pragma unroll
  for (int g0 = 0; g0 < 8; g0 += kBatch) {
    if (8 * g0 >= D) break;
    uint4 x[kBatch], t[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      if (8 * (g0 + k) < D) {
        x[k] = lds_u4(tile + sw128_off(r, g0 + k));
        t[k] = lds_u4(tab + sw128_off(r, g0 + k));
      }
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      if (8 * (g0 + k) < D) {
        const uint32_t xw[4] = {x[k].x, x[k].y, x[k].z, x[k].w};
        const uint32_t tw[4] = {t[k].x, t[k].y, t[k].z, t[k].w};
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 cs = Elt<__half>::unpack(tw[e]);
          const float2 v = Elt<T>::unpack(xw[e]);
          w[e] = Elt<T>::pack(v.x * cs.x - v.y * cs.y, v.y * cs.x + v.x * cs.y);
        }
        sts_u4(tile + sw128_off(r, g0 + k), make_uint4(w[0], w[1], w[2], w[3]));
      }
    }
  }
}

// Granule g (values 8g..8g+7) of a row of 64 f32 values, given as two
// 32-value halves, scaled and, with tab != 0, R^T-unrotated; packed to 16 bits.
template <typename T>
__device__ __forceinline__ uint4 row_granule_t(const float (&v0)[32], const float (&v1)[32], int g,
                                               float scale, uint32_t tab, int r) {
  uint32_t tw[4] = {0u, 0u, 0u, 0u};
  if (tab != 0u) {
    const uint4 t = lds_u4(tab + sw128_off(r, g));
    tw[0] = t.x; tw[1] = t.y; tw[2] = t.z; tw[3] = t.w;
  }
  float u[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int c = 8 * g + 2 * e;
    float a = (c < 32 ? v0[c & 31] : v1[c & 31]) * scale;
    float b = (c < 32 ? v0[(c + 1) & 31] : v1[(c + 1) & 31]) * scale;
    if (tab != 0u) {
      const float2 cs = Elt<__half>::unpack(tw[e]);
      const float a2 = a * cs.x + b * cs.y;
      b = b * cs.x - a * cs.y;
      a = a2;
    }
    u[2 * e] = a;
    u[2 * e + 1] = b;
  }
  return pack8<T>(u);
}

// Scale (and with tab != 0 R^T-unrotate) a row of 64 f32 values and store it
// to global memory.
template <typename T>
__device__ __forceinline__ void store_row_t(const float (&v0)[32], const float (&v1)[32], int D,
                                            float scale, uint32_t tab, int r, T* dst) {
#pragma unroll
  for (int g = 0; g < 8; ++g)
    if (8 * g < D) reinterpret_cast<uint4*>(dst)[g] = row_granule_t<T>(v0, v1, g, scale, tab, r);
}

// The same row written as row r of a one-chunk (128B-swizzled) shared tile,
// all 64 columns (a TMA store of the tile clips columns >= D).
template <typename T>
__device__ __forceinline__ void stage_row_t(const float (&v0)[32], const float (&v1)[32],
                                            float scale, uint32_t tab, int r, uint32_t tile) {
#pragma unroll
  for (int g = 0; g < 8; ++g) sts_u4(tile + sw128_off(r, g), row_granule_t<T>(v0, v1, g, scale, tab, r));
}

// Half h (columns [32 h, 32 h + 32), granules 4h..4h+3) of such a row, given
// as its 32 values, scaled, optionally R^T-unrotated, staged in a shared tile.
template <typename T>
__device__ __forceinline__ void stage_half_t(const float (&v)[32], int h, float scale,
                                             uint32_t tab, int r, uint32_t tile) {
#pragma unroll
  for (int gl = 0; gl < 4; ++gl) {
    const int g = 4 * h + gl;
    uint32_t tw[4] = {0u, 0u, 0u, 0u};
    if (tab != 0u) {
      const uint4 t = lds_u4(tab + sw128_off(r, g));
      tw[0] = t.x; tw[1] = t.y; tw[2] = t.z; tw[3] = t.w;
    }
    float u[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float a = v[8 * gl + 2 * e] * scale;
      float b = v[8 * gl + 2 * e + 1] * scale;
      if (tab != 0u) {
        const float2 cs = Elt<__half>::unpack(tw[e]);
        const float a2 = a * cs.x + b * cs.y;
        b = b * cs.x - a * cs.y;
        a = a2;
      }
      u[2 * e] = a;
      u[2 * e + 1] = b;
    }
    sts_u4(tile + sw128_off(r, g), pack8<T>(u));
  }
}

}  // namespace frsa

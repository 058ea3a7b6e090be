// Inline-PTX building blocks for the sm_100a kernels: mbarriers with bounded
// waits, TMA tile loads, tcgen05 (TMEM alloc, MMA, commit, loads) and the
// shared-memory matrix descriptors the tensor core reads.
//
// Every spin-wait here is bounded: after FRSA_WAIT_LIMIT_NS of global time the
// wait gives up, records FRSA_DEV_TIMEOUT in the device status word and sets the
// CTA-wide abort flag; every later wait in that CTA returns at once, so the CTA
// runs to its end, frees its TMEM and exits instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#ifndef FRSA_WAIT_LIMIT_NS
#define FRSA_WAIT_LIMIT_NS 2000000000ull  // 2 s: every legitimate wait is microseconds
#endif

namespace frsa {

// Device status word (0 = ok). Written only on a bounded-wait timeout. The
// library is a single translation unit, so this is its one definition.
__device__ int g_dev_status = 0;
enum : int { FRSA_DEV_TIMEOUT = 1, FRSA_DEV_SMEM = 2 };

// 1024-byte-aligned view of the dynamic shared memory, or nullptr (status
// FRSA_DEV_SMEM recorded) when the aligned struct would not fit the launch's
// dynamic allocation. The result is uniform across the CTA.
template <typename S>
__device__ __forceinline__ S* aligned_smem(uint8_t* raw) {
  uint32_t dyn;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
  const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(raw));
  const uint32_t pad = ((base + 1023u) & ~1023u) - base;
  if (pad + sizeof(S) > dyn) {
    if (threadIdx.x == 0) atomicExch(&g_dev_status, FRSA_DEV_SMEM);
    return nullptr;
  }
  return reinterpret_cast<S*>(raw + pad);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- tracing
// Trace builds (-DFRSA_TRACE) record %globaltimer at phase boundaries of the
// first 2048 CTAs, from thread FRSA_STAMP_TID (the first compute thread), into
// g_trace[cta * 64 + slot]; frsa_trace_copy reads them back. Normal builds
// compile the stamps away.
#ifndef FRSA_STAMP_TID
#define FRSA_STAMP_TID 64
#endif
#ifdef FRSA_TRACE
__device__ unsigned long long g_trace[2048 * 64];
// Per-iteration stamps of kernels that record them: [cta][iteration] times
// and event flags.
__device__ unsigned long long g_trace_it[2048 * 1024];
__device__ unsigned int g_trace_fl[2048 * 1024];
#define FRSA_STAMP(slot)                                                       \
  do {                                                                         \
    if (blockIdx.x < 2048 && threadIdx.x == FRSA_STAMP_TID)                    \
      ::frsa::g_trace[blockIdx.x * 64 + (slot)] = ::frsa::globaltimer();      \
  } while (0)
#define FRSA_STAMP_T(slot, tid)                                                \
  do {                                                                         \
    if (blockIdx.x < 2048 && threadIdx.x == (tid))                             \
      ::frsa::g_trace[blockIdx.x * 64 + (slot)] = ::frsa::globaltimer();      \
  } while (0)
#else
#define FRSA_STAMP(slot) \
  do {                   \
  } while (0)
#define FRSA_STAMP_T(slot, tid) \
  do {                          \
  } while (0)
#endif

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// try_wait: a thread whose phase is not complete waits in hardware for a
// short, implementation-defined time before the instruction returns false.
// (An explicit suspend-time hint was measured slower: with a 0.1 ms or 1 us
// hint the persistent kernels ran ~3 % longer, the waiting warps resuming
// later after the phase completed.)
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed. Returns false (and
// leaves the CTA in abort mode) if the wait timed out (FRSA_WAIT_LIMIT_NS) or
// the CTA was already aborting. The loop is one short PTX block so that the
// many wait sites of a kernel stay small in the instruction cache.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  uint32_t ok;
  asm volatile(
      "{\n\t"
      ".reg .pred p, q;\n\t"
      ".reg .u64 t0, t1;\n\t"
      ".reg .u32 ab;\n\t"
      "mov.u32 %0, 1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "@p bra WAIT_DONE;\n\t"
      "mov.u64 t0, %%globaltimer;\n\t"
      "WAIT_LOOP:\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "@p bra WAIT_DONE;\n\t"
      "ld.volatile.shared.u32 ab, [%3];\n\t"
      "setp.ne.u32 q, ab, 0;\n\t"
      "@q bra WAIT_FAIL;\n\t"
      "mov.u64 t1, %%globaltimer;\n\t"
      "sub.u64 t1, t1, t0;\n\t"
      "setp.lt.u64 q, t1, %4;\n\t"
      "@q bra WAIT_LOOP;\n\t"
      "WAIT_FAIL:\n\t"
      "mov.u32 %0, 0;\n\t"
      "WAIT_DONE:\n\t"
      "}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(smem_u32(const_cast<int*>(abort_flag))),
        "l"(static_cast<uint64_t>(FRSA_WAIT_LIMIT_NS))
      : "memory");
  if (ok) return true;
  if (*abort_flag == 0) {   // this wait timed out (not an abort raised elsewhere)
    *abort_flag = 1;
    atomicExch(&g_dev_status, FRSA_DEV_TIMEOUT);
  }
  return false;
}

// ---------------------------------------------------------------- global flags
// Acquire load / release store of a 32-bit flag in global memory (GPU scope).
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Drop a 128-byte line (128-byte aligned) from L2 without writing it back:
// for scratch whose contents are dead.
__device__ __forceinline__ void discard_l2_line(const void* p) {
  asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}

// Wait until the flag at `p` (written by another CTA) reaches `target`.
// Bounded like mbar_wait: gives up after FRSA_WAIT_LIMIT_NS, records
// FRSA_DEV_TIMEOUT and raises the CTA's abort flag; returns false then.
__device__ __forceinline__ bool flag_wait_geq(const int* p, int target, volatile int* abort_flag) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    __nanosleep(64);
    if (ld_acquire_gpu(p) >= target) return true;
    if (*abort_flag != 0) return false;
    if (globaltimer() - t0 > FRSA_WAIT_LIMIT_NS) {
      *abort_flag = 1;
      atomicExch(&g_dev_status, FRSA_DEV_TIMEOUT);
      return false;
    }
  }
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Named barrier among `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 3-D tiled load {x, y, z} -> shared, completion counted on `bar` in bytes.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// [B, H, N, D] tensors are addressed through 4-D maps {D, N, H, B} (any
// b/h/n strides, unit d stride); a kernel names a head by its flat index
// bh = b * H + h.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* tmap, uint64_t* bar, int x,
                                            int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void tma_load_bh(void* smem_dst, const void* tmap, uint64_t* bar, int x,
                                            int y, int bh, int H) {
  tma_load_4d(smem_dst, tmap, bar, x, y, bh % H, bh / H);
}
__device__ __forceinline__ void tma_prefetch_l2_bh(const void* tmap, int x, int y, int bh, int H) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(x), "r"(y), "r"(bh % H), "r"(bh / H)
               : "memory");
}

// 2-D tiled load global -> shared, completing on `bar` (transaction bytes).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Hint the tile {x, y, z} of a 3-D tensor map into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_3d(const void* tmap, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// Prefetch [p, p + bytes) into L2 (rounded out to 16-byte boundaries).
__device__ __forceinline__ void prefetch_l2_bytes(const void* p, uint32_t bytes) {
  const uint64_t a = reinterpret_cast<uint64_t>(p);
  const uint64_t lo = a & ~uint64_t(15), hi = (a + bytes + 15) & ~uint64_t(15);
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"(static_cast<uint32_t>(hi - lo))
               : "memory");
}

// Per-warpgroup register rebalancing (all 128 threads of a warpgroup execute it).
template <uint32_t R>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(R));
}
template <uint32_t R>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(R));
}

// 3-D tiled store shared -> {x, y, z} (elements outside the tensor are not
// written), as one bulk group of the issuing thread.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* smem_src, int x, int y,
                                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::
          "l"(reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_store_bh(const void* tmap, const void* smem_src, int x, int y,
                                             int bh, int H) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::
          "l"(reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(bh % H), "r"(bh / H)
      : "memory");
}
__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until the shared-memory sources of all committed store groups have been read.
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// 3-D tiled reduce-add shared -> {x, y, z} (f32 elements added at L2; elements
// outside the tensor are not touched), as one bulk group of the issuing thread.
__device__ __forceinline__ void tma_reduce_add_3d(const void* tmap, const void* smem_src, int x,
                                                  int y, int z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::
          "l"(reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// Wait until all committed bulk groups of this thread have completed (their
// global writes done), then order them before later generic-proxy accesses.
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: writes the base address to *slot (shared). Whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 or f16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16. A is M x K with row m in
// TMEM lane m and two 16-bit K elements per 32-bit column (K = 16 per
// instruction = 8 columns).
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05 ops of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Load 32 consecutive f32 columns of this thread's TMEM lane.
// 8 consecutive 32-bit columns of this thread's TMEM lane (32x32b.x8).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Load 16 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor for a 128-byte-swizzled canonical layout.
//   bits  0-13 start address >> 4, 16-29 leading byte offset >> 4,
//   bits 32-45 stride byte offset >> 4, bits 46-47 version (1 on sm_100),
//   bits 61-63 layout (2 = 128B swizzle).
// K-major operand: rows of 128 B (64 16-bit elements), 8-row atoms 1024 B apart
// (SBO); one 16-element K step = +32 B on the start address.
// MN-major operand: 64 contiguous MN elements per 128 B row, rows are K; LBO =
// byte distance between 64-element MN blocks, SBO = distance between 8-row K groups.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f32 accumulation.
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (0 = f16, 1 = bf16),
//   bit 15 A major (1 = MN), bit 16 B major, bits 17-22 N >> 3, bits 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------- shared-space access
// Explicit shared-state-space loads and stores. Unlike generic pointer
// accesses, the compiler knows these cannot alias global memory, so global
// loads around them keep their freedom to be hoisted and batched. They carry
// no memory clobber, so ordinary global loads may still move across them, but
// they are volatile: they stay ordered after the mbarrier waits and named
// barriers (also volatile asm) that make the shared data valid.
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float2 lds_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v));
}
__device__ __forceinline__ void sts_u4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w));
}
__device__ __forceinline__ void sts_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w));
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16-bit element traits: pack two f32 into one 32-bit word (first value in
// the low half) and back, in registers only.
template <typename T>
struct Elt;
template <>
struct Elt<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    uint32_t u;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(b), "f"(a));
    return u;
  }
  __device__ static __forceinline__ float2 unpack(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
};
template <>
struct Elt<__half> {
  static constexpr bool kBf16 = false;
  __device__ static __forceinline__ uint32_t pack(float a, float b) {
    uint32_t u;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(b), "f"(a));
    return u;
  }
  __device__ static __forceinline__ float2 unpack(uint32_t w) {
    float lo, hi;
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "cvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
        : "=f"(lo), "=f"(hi)
        : "r"(w));
    return make_float2(lo, hi);
  }
};

// Byte offset of 16-byte granule `g` (0..7) of row `r` inside a 128B-swizzled
// tile whose rows are 128 B and whose base is 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t g) {
  return r * 128u + ((g ^ (r & 7u)) << 4);
}

}  // namespace frsa

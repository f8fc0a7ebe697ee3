// Blackwell (sm_100a) building blocks for the batched GEMMs: mbarriers, TMA
// tile loads, tensor memory (TMEM) and tcgen05.mma with 8-bit integer inputs.
#pragma once
#include <cuda.h>

#include <cstdint>

namespace q4 {
namespace umma {

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarriers ---------------------------------------------------------------
__device__ __forceinline__ void bar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}
__device__ __forceinline__ bool bar_try_wait(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of the given parity; gives up after `limit_ns` and
// returns false (the caller records the error and winds down).  (A variant
// that passed a suspend-time hint to try_wait slowed the cluster attention's
// ring by a quarter: the plain try_wait loop stays.)
__device__ __forceinline__ bool bar_wait(uint64_t* b, unsigned parity, uint64_t limit_ns = 200000000ull) {
  if (bar_try_wait(b, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (bar_try_wait(b, parity)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > limit_ns) return false;
  }
}

// ---- TMA ---------------------------------------------------------------------
__device__ __forceinline__ void prefetch_map(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2-D tile load into this CTA's shared memory, completion counted on bar.
__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* m, int x, int y, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_addr(b))
      : "memory");
}

// ---- tensor memory -----------------------------------------------------------
// Column allocation by one full warp; the TMEM address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x N consecutive 32-bit columns: thread i of the warp receives
// lane (sub-partition base + i), columns col .. col + N - 1.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, int32_t* r);
template <>
__device__ __forceinline__ void tmem_ld<1>(uint32_t taddr, int32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<2>(uint32_t taddr, int32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, int32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, int32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, int32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Any N in 1..31 as a sum of the power-of-two shapes.
template <int N>
__device__ __forceinline__ void tmem_ld_any(uint32_t taddr, int32_t* r) {
  if constexpr (N >= 16) {
    tmem_ld<16>(taddr, r);
    tmem_ld_any<N - 16>(taddr + 16, r + 16);
  } else if constexpr (N >= 8) {
    tmem_ld<8>(taddr, r);
    tmem_ld_any<N - 8>(taddr + 8, r + 8);
  } else if constexpr (N >= 4) {
    tmem_ld<4>(taddr, r);
    tmem_ld_any<N - 4>(taddr + 4, r + 4);
  } else if constexpr (N >= 2) {
    tmem_ld<2>(taddr, r);
    tmem_ld_any<N - 2>(taddr + 2, r + 2);
  } else if constexpr (N == 1) {
    tmem_ld<1>(taddr, r);
  }
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- tcgen05.mma -------------------------------------------------------------
// Shared-memory matrix descriptor: K-major tile whose rows are 128 bytes,
// written by TMA with 128-byte swizzling (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu)   // start address
         | ((uint64_t)1 << 16)                // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)      // stride byte offset: 8 rows x 128 B
         | ((uint64_t)1 << 46)                // descriptor version (sm_100)
         | ((uint64_t)2 << 61);               // 128-byte swizzle
}

// Instruction descriptor of kind::i8: s32 accumulator, A signed, B unsigned,
// both K-major, M x N.
__host__ __device__ constexpr uint32_t i8_idesc(int M, int N) {
  return (2u << 4) | (1u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// The same with the signedness of each operand chosen (u8 or s8).
__host__ __device__ constexpr uint32_t i8_idesc_ab(int M, int N, bool a_signed, bool b_signed) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] x B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
// The same with the accumulate flag fixed: D = A B (init) or D += A B (acc).
// A descriptor's start-address field is (address >> 4) in its low 14 bits, so
// the descriptor of a tile at a 16-byte multiple `off` past another is that
// descriptor + off / 16 (shared-memory addresses stay below 2^18).
__device__ __forceinline__ void mma_i8_init(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, 0, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%4, %4, %4, %4}, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0)
      : "memory");
}
__device__ __forceinline__ void mma_i8_acc(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.eq.b32 p, 0, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%4, %4, %4, %4}, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0)
      : "memory");
}
// Arrive on bar once every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void mma_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(b))
               : "memory");
}

// ---- clusters ----------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_st64(uint32_t caddr, int64_t v) {
  asm volatile("st.shared::cluster.b64 [%0], %1;" ::"r"(caddr), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t cluster_ld64(uint32_t caddr) {
  int64_t v;
  asm volatile("ld.shared::cluster.b64 %0, [%1];" : "=l"(v) : "r"(caddr) : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace umma
}  // namespace q4

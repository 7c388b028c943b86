// ptx.cuh -- sm_100a primitives used by the ltx25 kernels: mbarriers with
// bounded waits, TMA tile loads (each CTA fetches its own tiles), tcgen05 TMEM
// allocation / MMA / load / store, and the UMMA descriptors.
//
// Every wait here gives up after a wall-clock bound (kWaitNs) and reports
// failure instead of spinning forever; the kernels turn that into an error
// flag the host reads, and exit cleanly.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ltx {

// ~2 s: far beyond any legitimate wait in these kernels, short enough that
// a broken pipeline returns an error instead of holding the GPU.
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id()
{
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ---- mbarrier --------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes)
{
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with parity `parity` to complete.  Returns false when
// `abort` was raised by another role or the wall-clock bound ran out (the
// latter also raises `abort` and records `code` in `*err`).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort, int* err,
                                          int code)
{
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      *abort = 1;
      if (err != nullptr) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// ---- TMA ---------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const void* map)
{
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 2-D tiled load into this CTA's shared memory, completing on `bar`.
// (x, y) are element coordinates; x * element size is a multiple of 16 B at
// every call site.
__device__ __forceinline__ void tma_load_2d(const void* map, uint64_t* bar,
                                            void* dst, int x, int y)
{
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---- tcgen05 -------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols)
{
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16 in, f32 acc).
__device__ __forceinline__ void umma_f16_ss(uint32_t d, uint64_t a, uint64_t b,
                                            uint32_t idesc, uint32_t acc)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16.
__device__ __forceinline__ void umma_f16_ts(uint32_t d, uint32_t a_tmem,
                                            uint64_t b, uint32_t idesc,
                                            uint32_t acc)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// D(tmem, s32) (+)= A(smem) * B(smem), kind::i8.
__device__ __forceinline__ void umma_i8_ss(uint32_t d, uint64_t a, uint64_t b,
                                           uint32_t idesc, uint32_t acc)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op this thread issued so far has
// completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld()
{
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st()
{
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (base lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, "
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, "
      "%22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr,
                                          const uint32_t (&r)[32])
{
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, "
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, "
      "%22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}

// ---- UMMA descriptors (CUTLASS cute/arch/mma_sm100_desc.hpp layout) ----

// Shared-memory matrix descriptor for a K-major operand whose rows are 128
// bytes, written by TMA with SWIZZLE_128B: 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc_k128_sw128(uint32_t saddr)
{
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);       // start address
  d |= (uint64_t)(16 >> 4) << 16;                // LBO (unused for SW128 K)
  d |= (uint64_t)(1024 >> 4) << 32;              // SBO: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                        // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16 with bf16 A/B, f32 accumulate, both
// operands K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N)
{
  return (1u << 4)                       // c_format = F32
         | (1u << 7)                     // a_format = BF16
         | (1u << 10)                    // b_format = BF16
         | ((uint32_t)(N >> 3) << 17)    // n_dim
         | ((uint32_t)(M >> 4) << 24);   // m_dim
}

// Instruction descriptor: kind::i8, A signed, B signed, s32 accumulate.
__host__ __device__ constexpr uint32_t idesc_s8(int M, int N)
{
  return (2u << 4)                       // c_format = S32
         | (1u << 7)                     // a_format = signed 8-bit
         | (1u << 10)                    // b_format = signed 8-bit
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads)
{
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- cta_group::2 (two SMs per MMA) -----------------------------------------

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols)
{
  asm volatile(
      "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

// D (+)= A(tmem) * B(smem), M = 256 across the CTA pair: each CTA's TMEM
// holds its 128 rows of A and D, each CTA's shared memory its half of B at
// the same offset.  Issued by the leader CTA only.
__device__ __forceinline__ void umma_f16_ts_pair(uint32_t d, uint32_t a_tmem,
                                                 uint64_t b, uint32_t idesc,
                                                 uint32_t acc)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// D (+)= A(smem) * B(smem), M = 256 across the CTA pair: each CTA's shared
// memory holds its 128 rows of A and its half of B at the same offsets, each
// CTA's TMEM its 128 rows of D.  Issued by the leader CTA only.
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d, uint64_t a, uint64_t b,
                                                 uint32_t idesc, uint32_t acc)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive once on the mbarrier at shared::cluster address `caddr` (this CTA's
// or the peer's) when the pair MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t caddr)
{
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(caddr)
      : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted
// on the mbarrier at shared::cluster address `cbar` -- the leader CTA's.
__device__ __forceinline__ void tma_load_2d_pair(const void* map, uint32_t cbar,
                                                 void* dst, int x, int y)
{
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::"
      "complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(cbar), "r"(x), "r"(y)
      : "memory");
}

// Arrive on an mbarrier in another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr)
{
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr)
               : "memory");
}

// ---- thread-block clusters (distributed shared memory) -------------------

__device__ __forceinline__ uint32_t cluster_ctarank()
{
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster arrives, then waits.  Writes to
// shared memory before the barrier are visible to peers after it.
__device__ __forceinline__ void cluster_sync_all()
{
  asm volatile(
      "barrier.cluster.arrive.release;\n\t"
      "barrier.cluster.wait.acquire;" ::
          : "memory");
}

// The shared::cluster address of `saddr` (a shared::cta address) in CTA
// `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank)
{
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(r)
               : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t caddr)
{
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(caddr)
               : "memory");
  return v;
}

}  // namespace ltx

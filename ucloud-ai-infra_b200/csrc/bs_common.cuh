// Device primitives for the sm_100a block-scaled FP8 kernels: mbarriers with bounded waits,
// TMA tile loads (no cluster multicast anywhere), tcgen05 MMA / TMEM access and the UMMA
// descriptors for K-major 128-byte-swizzled operands.
//
// Every wait in this library is bounded by wall time (%globaltimer). When a bound runs out the
// waiting thread records an error code in the library's status word, raises the CTA's abort
// flag and returns false; the caller leaves its loop, drains what it has in flight (again with
// a bound) and the CTA frees its TMEM before it exits. No wait can spin forever and no kernel
// traps.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace bs {

// ---- error codes shared with the host (include/bs_fp8.h mirrors these values) ----
enum : int {
  kOk = 0,
  kErrTimeoutFull = 101,     // MMA issuer waited too long for a TMA stage
  kErrTimeoutEmpty = 102,    // TMA producer waited too long for a free stage
  kErrTimeoutPFull = 103,    // promotion warps waited too long for an MMA partial
  kErrTimeoutPEmpty = 104,   // MMA issuer waited too long for a free TMEM partial buffer
  kErrTimeoutDrain = 105,    // teardown waited too long for in-flight copies / MMAs
  kErrTimeoutPeer = 106,     // tensor-parallel reduce: a peer rank's CTA did not arrive in time
  kErrTimeoutSelftest = 199, // the self-test wait ran out, as it is meant to
};

// Bound on every mbarrier wait: 4 s of wall time. No legitimate wait in these kernels lasts
// longer than a few microseconds.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Waits for the phase of `bar` with the given parity to complete. Gives up after `limit_ns`
// (or as soon as another role of the CTA raised *abort), records `code` in *status and
// returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                          int code, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*abort) return false;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(status, 0, code);
        *abort = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA (per-CTA, never multicast)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box into shared memory; completion is signalled on `bar` as
// transaction bytes. `policy` is an L2 cache policy made by createpolicy.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Pair form (cta_group::2, no multicast): the box lands in this CTA's shared memory and its bytes
// are counted on the barrier at shared::cluster address `bar_cluster`, which may be the peer CTA's.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Brings one box of a tensor into L2 without waiting for it (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// Programmatic dependent launch. Every library kernel is launched allowed to start before the
// previous kernel on its stream has finished; grid_dep_wait() returns once the grids it depends on
// have completed and their writes are visible, so every global access of a thread that could
// depend on them comes after it (an L2 prefetch cannot observe stale data and may precede it).
// grid_dep_launch() lets the next such launch start its prologue on SMs this grid leaves free.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// 2-D tiled store of one box from shared memory (rows outside the tensor are not written),
// tracked by the issuing thread's bulk async-group. Generic-proxy writes to `src` must be
// followed by fence_proxy_async_smem() and a barrier before the store is issued.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Returns once every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> f32. Issued by one thread.
__device__ __forceinline__ void mma_e4m3(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- CTA pairs (cluster of 2, cta_group::2)
// A pair of CTAs on the two SMs of a TPC computes one 256-row tile: each CTA holds its own 128 A rows
// and half of the weight rows in its shared memory, the leader (rank 0) issues the MMAs, and each CTA's
// TMEM receives its 128 rows of the result. Loads are plain per-CTA TMA loads (never multicast).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}
// Relaxed remote arrival: the count only, no memory ordering. Hands a TMEM buffer back after
// tcgen05.wait::ld (the loads have completed; nothing this thread wrote needs to be seen).
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Tensor-parallel reductions through NVSwitch: `mc` is a multicast address (the same buffer mapped on
// every rank); the switch adds the values into each rank's copy (bf16 arithmetic, any order of ranks).
__device__ __forceinline__ void multimem_add_bf16x8(void* mc, const uint4& v) {
  asm volatile("multimem.red.relaxed.sys.global.add.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void multimem_add_bf16x2(void* mc, uint32_t v) {
  asm volatile("multimem.red.relaxed.sys.global.add.bf16x2 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}
// Orders this thread's earlier memory operations, multimem ones included, before its later ones at
// system scope.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Busy-waits `ns` nanoseconds of wall time.
__device__ __forceinline__ void pause_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) {
  }
}
// Every thread of both CTAs; orders all earlier shared-memory and barrier work cluster-wide.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (both CTAs' TMEM, 128 rows each) (+)= A (each CTA's own rows) * [B half of CTA 0; B half of CTA 1]^T.
__device__ __forceinline__ void mma_e4m3_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` in every CTA of `cta_mask` when this thread's pair MMAs so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}


__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit values: thread i of the warp receives lane (base+i),
// columns col..col+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
      "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]),
        "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]),
        "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]),
        "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]),
        "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}

// Issues loads of N consecutive TMEM columns (N a multiple of 4, at most 128) of this warp's 32
// lanes into v[0..N), largest pieces first, all in flight together; the caller waits once.
template <int N, int OFF = 0>
__device__ __forceinline__ void tmem_ld_run(uint32_t taddr, uint32_t* v) {
  static_assert(N % 4 == 0 && N >= 0, "column run");
  if constexpr (N >= 64) {
    tmem_ld64(taddr + OFF, *reinterpret_cast<uint32_t(*)[64]>(v + OFF));
    tmem_ld_run<N - 64, OFF + 64>(taddr, v);
  } else if constexpr (N >= 32) {
    tmem_ld32(taddr + OFF, *reinterpret_cast<uint32_t(*)[32]>(v + OFF));
    tmem_ld_run<N - 32, OFF + 32>(taddr, v);
  } else if constexpr (N >= 16) {
    tmem_ld16(taddr + OFF, *reinterpret_cast<uint32_t(*)[16]>(v + OFF));
    tmem_ld_run<N - 16, OFF + 16>(taddr, v);
  } else if constexpr (N >= 8) {
    tmem_ld8(taddr + OFF, *reinterpret_cast<uint32_t(*)[8]>(v + OFF));
    tmem_ld_run<N - 8, OFF + 8>(taddr, v);
  } else if constexpr (N >= 4) {
    tmem_ld4(taddr + OFF, *reinterpret_cast<uint32_t(*)[4]>(v + OFF));
  }
}

// Shared-memory matrix descriptor of a K-major operand laid out by TMA with 128-byte swizzle:
// rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N. The tile base must be
// 1024-byte aligned; stepping along K inside the 128-byte row is a plain start-address offset.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address, 16-byte units
  d |= static_cast<uint64_t>(1) << 16;                   // leading byte offset (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;           // stride byte offset: next 8-row group
  d |= static_cast<uint64_t>(1) << 46;                   // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;                   // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f8f6f4: A = B = e4m3, D = f32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
  return (1u << 4)                                   // D format f32
         | (0u << 7) | (0u << 10)                    // A, B: e4m3
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// ---------------------------------------------------------------- register split
// Warp-specialised kernels launch every thread at the same register count; the warpgroup that
// only issues TMA / MMA instructions then gives registers back (setmaxnreg.dec) and the
// promotion warpgroups take them (setmaxnreg.inc). An increase draws on the registers the block
// was launched with, so a split must add up exactly to threads x launch registers, and the host
// refuses to launch a kernel whose build does not have exactly the launch count it was designed
// for (any other count would make the increase wait forever).
template <int kThreads_, int kLaunch_, int kProducer_, int kConsumer_>
struct RegSplit {
  static constexpr int kThreads = kThreads_;
  static constexpr int kLaunch = kLaunch_;
  static constexpr int kProducer = kProducer_;    // one warpgroup of 128 threads
  static constexpr int kConsumer = kConsumer_;    // every other thread
  static_assert(128 * kProducer + (kThreads - 128) * kConsumer == kThreads * kLaunch,
                "register split must use exactly the registers the block was launched with");
  static_assert(kLaunch % 8 == 0 && kProducer % 8 == 0 && kConsumer % 8 == 0, "register counts in steps of 8");
};

template <int N>
__device__ __forceinline__ void regs_increase() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_decrease() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Keeps the compiler from hoisting loads across this point (bounds live registers).
__device__ __forceinline__ void compiler_fence() { asm volatile("" ::: "memory"); }

// ---------------------------------------------------------------- stage counters
// Built only with -DBS_TRACE (a profiling build; the product build compiles these to nothing).
// Each role accumulates clock64() cycles per pipeline segment in registers and adds them to
// g_bs_trace once at the end, so the counters cost nothing inside the loops but two clock reads.
#ifdef BS_TRACE
__device__ unsigned long long g_bs_trace[64];
#define BS_TR_DECL(n)        \
  long long bs_tr[n] = {0};  \
  const long long bs_tr_t0 = clock64(); \
  long long bs_tr_mark = bs_tr_t0
#define BS_TR_MARK() (bs_tr_mark = clock64())
#define BS_TR_ADD(i)                   \
  do {                                 \
    const long long bs_tr_now = clock64(); \
    bs_tr[i] += bs_tr_now - bs_tr_mark;    \
    bs_tr_mark = bs_tr_now;                \
  } while (0)
#define BS_TR_FLUSH(base, n)                                                                    \
  do {                                                                                          \
    for (int bs_tr_i = 0; bs_tr_i < (n); ++bs_tr_i)                                             \
      atomicAdd(&g_bs_trace[(base) + bs_tr_i], static_cast<unsigned long long>(bs_tr[bs_tr_i])); \
    atomicAdd(&g_bs_trace[(base) + (n)], static_cast<unsigned long long>(clock64() - bs_tr_t0)); \
    atomicAdd(&g_bs_trace[(base) + (n) + 1], 1ull);                                             \
  } while (0)
#else
#define BS_TR_DECL(n) \
  do {                \
  } while (0)
#define BS_TR_MARK() \
  do {               \
  } while (0)
#define BS_TR_ADD(i) \
  do {               \
  } while (0)
#define BS_TR_FLUSH(base, n) \
  do {                       \
  } while (0)
#endif

// ---------------------------------------------------------------- misc
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float ldg_f32(const float* p) { return __ldg(p); }

// ---------------------------------------------------------------- packed fp32 pairs
// Accumulators are kept as pairs in 64-bit registers so the promotion runs on the packed
// fma.rn.f32x2 (sm_100): each lane is an ordinary fma.rn.f32, so results are bit-identical to
// two scalar fmaf calls while the instruction count halves.
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }

// acc.{lo,hi} = fma({p0, p1}, s.{lo,hi}, acc.{lo,hi}), round to nearest even per lane.
__device__ __forceinline__ void ffma2(uint64_t& acc, uint32_t p0, uint32_t p1, uint64_t s) {
  asm("{\n\t.reg .b64 p;\n\tmov.b64 p, {%1, %2};\n\tfma.rn.f32x2 %0, p, %3, %0;\n\t}"
      : "+l"(acc)
      : "r"(p0), "r"(p1), "l"(s));
}

// Two floats -> two e4m3 bytes (round to nearest even, saturate to +-448), low byte = a.
__device__ __forceinline__ uint32_t f2_to_e4m3x2(float a, float b) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// SiLU(g) * u in fp32: g / (1 + e^-g) * u, with the hardware exponential and a fast divide, as
// the reference's fused kernel does with ex2.approx / rcp.approx (patches/fp8_hand_sm89.py:538-539).
// Relative error stays within a few fp32 ulp; for g -> -inf the divisor overflows to +inf and
// the fast divide returns 0, the correct limit.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdividef(g, 1.0f + __expf(-g)), u);
}

// ---------------------------------------------------------------- warp max of N values per lane
// Max over the 32 lanes of each of v[0..N) (unsigned; non-negative floats order like their bits).
// While the count is even, each exchange halves it: the lanes with bit OFF set keep the upper half
// of the values and send the lower half to their partner, so N values cost N/2 + N/4 + ...
// shuffles instead of 5*N. An odd remainder finishes with plain xor reductions. Afterwards lane
// L holds the maxima of tokens warp_max_base<N, 16>(L) + [0, warp_max_count<N, 16>()), and the
// lanes that differ only in bits of warp_max_dup_mask<N, 16>() hold identical copies.
template <int N, int OFF>
__device__ __forceinline__ void warp_max_halving(uint32_t* v, int lane) {
  if constexpr (OFF > 0) {
    if constexpr (N % 2 == 0) {
      const bool upper = (lane & OFF) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        const uint32_t send = upper ? v[i] : v[N / 2 + i];
        const uint32_t keep = upper ? v[N / 2 + i] : v[i];
        v[i] = max(keep, __shfl_xor_sync(0xffffffffu, send, OFF));
      }
      warp_max_halving<N / 2, OFF / 2>(v, lane);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = max(v[i], __shfl_xor_sync(0xffffffffu, v[i], OFF));
      warp_max_halving<N, OFF / 2>(v, lane);
    }
  }
}
template <int N, int OFF>
__host__ __device__ constexpr int warp_max_count() {
  if constexpr (OFF == 0) return N;
  else if constexpr (N % 2 == 0) return warp_max_count<N / 2, OFF / 2>();
  else return warp_max_count<N, OFF / 2>();
}
template <int N, int OFF>
__host__ __device__ constexpr int warp_max_dup_mask() {
  if constexpr (OFF == 0) return 0;
  else if constexpr (N % 2 == 0) return warp_max_dup_mask<N / 2, OFF / 2>();
  else return OFF | warp_max_dup_mask<N, OFF / 2>();
}
template <int N, int OFF>
__device__ __forceinline__ int warp_max_base(int lane) {
  if constexpr (OFF == 0) return 0;
  else if constexpr (N % 2 == 0) return ((lane & OFF) ? N / 2 : 0) + warp_max_base<N / 2, OFF / 2>(lane);
  else return warp_max_base<N, OFF / 2>(lane);
}

}  // namespace bs

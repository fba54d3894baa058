// Tensor-parallel sum of the ranks' bf16 partials through the NVSwitch, in place.
//
// Every rank's down_proj partial [rows, cols] sits in its own copy of a symmetric buffer that has an
// NVSwitch multicast mapping. Rank r owns the r-th 1/world of the buffer's 16-byte vectors: it reads each
// owned vector reduced over all ranks with one multimem.ld_reduce (the switch adds the world bf16 values with
// fp32 accumulation and rounds the sum to bf16 once) and writes the sum into every rank's copy with one
// multimem.st. Per GPU that is about (world-1)/world of the buffer out and the same in, whatever the world
// size, and every copy ends up with the same bytes (one read-reduce per vector, broadcast).
//
// Ordering. CTA b of every rank meets CTA b of every other rank twice, through a flag array in a second
// symmetric buffer with a multicast mapping, flags[phase][b][rank] (uint32; the values are the launch's epoch,
// which grows by one per launch, so nothing is ever reset):
//   phase 0, before reading: the partial of this rank is complete (the launch is stream-ordered after the GEMM
//            that wrote it); thread 0 publishes that with a release store of the epoch to every rank's
//            flags[0][b][rank], then waits until flags[0][b][q] >= epoch for every q;
//   phase 1, after writing:  the same with flags[1][...] once every thread's multimem stores are issued and
//            fenced, so that no rank's kernel ends before every rank's stores into its copy are done, and no
//            rank reads or overwrites its copy while a peer may still read it.
// CTA b of every rank covers the same share of its rank's range, so waiting on CTA b of every rank is enough:
// when all CTAs of a rank's launch have passed phase 1, every rank's every store into its copy is done.
// Each wait is bounded (limit_ns); a CTA that gives up records kErrTimeoutPeer in the status word and returns without
// signalling the next phase, so the peers' waits run out too and every rank reports the error.
#pragma once
#include "bs_common.cuh"

namespace bs {

constexpr int kTpThreads = 512;
constexpr int kTpMaxCtas = 256;     // flag words per phase and rank
constexpr int kTpUnroll = 4;        // 16-byte vectors in flight per thread

__device__ __forceinline__ uint4 multimem_ld_reduce_bf16x8(uint64_t mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void multimem_st_bf16x8(uint64_t mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void multimem_st_release_u32(uint64_t mc, uint32_t v) {
  asm volatile("multimem.st.release.sys.global.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One meeting of CTA blockIdx.x of every rank (see the file comment). Returns false after a timeout.
__device__ __forceinline__ bool tp_meet(uint32_t* flags, uint64_t flags_mc, int phase, int rank, int world,
                                        uint32_t epoch, uint64_t limit_ns, int* status) {
  const int slot = (phase * kTpMaxCtas + blockIdx.x) * world;
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();  // this CTA's earlier stores (multimem ones included) before the flag
    multimem_st_release_u32(flags_mc + 4ull * (slot + rank), epoch);
  }
  bool ok = true;
  if (static_cast<int>(threadIdx.x) < world) {
    const uint32_t* f = flags + slot + threadIdx.x;
    ok = static_cast<int>(ld_acquire_sys_u32(f) - epoch) >= 0;
    if (!ok) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t spins = 1;; ++spins) {
        if (static_cast<int>(ld_acquire_sys_u32(f) - epoch) >= 0) {
          ok = true;
          break;
        }
        if ((spins & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) break;
      }
    }
    if (!ok) atomicCAS(status, 0, kErrTimeoutPeer);
  }
  return __syncthreads_and(ok) != 0;
}

// data_mc: multicast address of the bf16 buffer (nvec 16-byte vectors); flags / flags_mc: this rank's flag
// words and the flag buffer's multicast address.
__global__ void __launch_bounds__(kTpThreads) k_tp_reduce_switch(uint64_t data_mc, uint32_t* flags, uint64_t flags_mc,
                                                                 long long nvec, int rank, int world, uint32_t epoch,
                                                                 uint64_t limit_ns, int* status) {
  if (!tp_meet(flags, flags_mc, 0, rank, world, epoch, limit_ns, status)) return;
  const long long v0 = nvec * rank / world, v1 = nvec * (rank + 1) / world;
  const long long per = (v1 - v0 + gridDim.x - 1) / gridDim.x;
  const long long c0 = v0 + per * blockIdx.x;
  const long long c1 = c0 + per < v1 ? c0 + per : v1;
  constexpr long long kStep = static_cast<long long>(kTpThreads) * kTpUnroll;
  for (long long base = c0; base < c1; base += kStep) {
    uint4 v[kTpUnroll];
#pragma unroll
    for (int i = 0; i < kTpUnroll; ++i) {
      const long long idx = base + threadIdx.x + static_cast<long long>(kTpThreads) * i;
      if (idx < c1) v[i] = multimem_ld_reduce_bf16x8(data_mc + 16ull * idx);
    }
#pragma unroll
    for (int i = 0; i < kTpUnroll; ++i) {
      const long long idx = base + threadIdx.x + static_cast<long long>(kTpThreads) * i;
      if (idx < c1) multimem_st_bf16x8(data_mc + 16ull * idx, v[i]);
    }
  }
  __syncthreads();
  tp_meet(flags, flags_mc, 1, rank, world, epoch, limit_ns, status);
}

}  // namespace bs

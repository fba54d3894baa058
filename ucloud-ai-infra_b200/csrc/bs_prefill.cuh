// Prefill-size block-scaled FP8 GEMM for sm_100a (M > 128 rows).
//
// Computes, per output tile of 128 rows x 256 columns,
//     C[m, n] = sum_kb  P_kb[m, n] * (As[m, kb] * Bs[n / 128, kb])
// where P_kb is the fp32 product of one 128-wide K block of e4m3 activations and e4m3 weights.
// This is the arithmetic of the reference kernel (patches/fp8_hand_sm89.py:189-199 and
// :275-280): one fp32 partial per 128-K block, the scale product a_s * b_s rounded once, then
// C = fma(partial, scale, C). The reference keeps the partial in mma.sync registers; here it
// comes from tcgen05.mma into TMEM and is promoted by CUDA-core warps.
//
// CTA layout (384 threads, one persistent CTA per SM):
//   warps 0-7  promotion + epilogue. Warp w reads TMEM lanes 32*(w%4)..+31 (one tile row per
//              thread) and columns 128*(w/4)..+127: one 128-wide weight block (plain), so the scale
//              product is one scalar per thread per K block, or 64 gate and 64 up columns (fused), two.
//   warp 8     TMA producer: A box 128x128 and 256 weight rows x 128 bytes per K block (two 128-row
//              boxes; fused: four 64-row boxes).
//   warp 9     TMEM allocator + MMA issuer: 4 x tcgen05.mma (M=128, N=256, K=32) per K block
//              into one of two TMEM partial buffers (2 x 256 columns = all 512).
//   warps 10-11 idle; warps 8-11 form the warpgroup that hands its registers to warps 0-7
//              (setmaxnreg 40 / 232), since each promotion thread keeps 128 fp32 accumulators.
// The partial buffers are double-buffered, so the tensor core computes block kb+1 while the
// promotion warps fold block kb into their register accumulators.
//
// FUSED=true is the gate_up + SiLU*up + per-token-group quant kernel (reference
// patches/fp8_hand_sm89.py:314-583): the 256 MMA columns are [gate 0-63 | up 0-63 | gate 64-127 |
// up 64-127] of gate block j and up block j + I/128 (I = N/2), loaded as 64-row weight boxes, so each
// promotion thread holds gate and up of the same 64 output columns and forms y without any exchange; the
// two warpgroups meet only to take the 128-wide quant group's amax:
//   y = silu(g) * u;  scale = max(amax|y|, 1e-10) / 448;  q = sat_e4m3(y * (1 / scale)).
#pragma once
#include <type_traits>

#include "bs_common.cuh"

namespace bs {

struct GemmParams {
  int M, N, K, KB;   // N: output features (plain) or gate+up rows, 2*I (fused)
  int ldc;           // plain: row stride of the output, in elements
  int b_tiled;       // 1: weights in tile-first layout [N/128][K/128][128][128]; 0: row-major [N, K]
  int out_f32;       // plain: write fp32 instead of bf16
  int group_m;       // prefill raster: M tiles per group
  const float* As;   // [M, KB] activation group scales
  const float* Bs;   // [N/128, KB] weight block scales
  void* out;         // plain: C [M, ldc]; fused: Q e4m3 [M, I]
  float* qs;         // fused: Qs [M, I/128]
  float* ws;         // decode split-K and stream-K prefill partials
  int* cnt;          // their arrival counters, one per tile, zero between launches
  int* status;       // library status word
  int out_mc;        // plain bf16: `out` is a multicast address; tiles are added into every rank's copy
};

template <bool FUSED, bool PAIR = false>
struct PrefillCfg {
  using Regs = RegSplit<384, 168, 40, 232>;
  static constexpr int kThreads = Regs::kThreads;
  static constexpr int kStages = PAIR ? 6 : 4;
  static constexpr int kABytes = 128 * 128;
  static constexpr int kBBytes = (PAIR ? 128 : 256) * 128;  // a pair CTA holds half of the weight rows
  static constexpr int kStageBytes = kABytes + kBBytes;
  // fused: the two warpgroups' amax halves per row; plain: a 4 KB row-transpose buffer per promotion warp
  // (multicast output)
  static constexpr int kXchBytes = FUSED ? 128 * 2 * 4 : 8 * 4096;
  static constexpr int kBarOff = kStages * kStageBytes + kXchBytes;
  static constexpr int kSmemBytes = kBarOff + 256 + 1024;  // barriers, then slack for 1 KB alignment
  static constexpr int kTmemCols = 512;
  static constexpr int kRows = PAIR ? 256 : 128;  // output rows per tile
};

// Tile index -> (m tile, n tile), grouped so that CTAs running together share A and B tiles in L2: groups of
// group_m M tiles, and inside a group consecutive tiles walk down one weight column tile, so the group's
// activation rows stay in L2 while the weight tiles stream past them (with every M tile in one group, each
// weight tile is fetched from HBM once).
__device__ __forceinline__ void prefill_tile_coords(int tile, int num_m, int num_n, int group_m, int& tm, int& tn) {
  const int per_group = group_m * num_n;
  const int g = tile / per_group;
  const int first_m = g * group_m;
  const int gm = min(num_m - first_m, group_m);
  const int in = tile - g * per_group;
  tm = first_m + in % gm;
  tn = in / gm;
}

// Segment i (0, 1, ...) of one CTA's work: tile `tile`, K blocks [kb0, kb1). Whole tiles c, c + G, ... without
// stream-K; with it, the contiguous (tile, K block) units [c*U/G, (c+1)*U/G) of U = num_tiles * KB cut at tile
// boundaries, so every CTA streams the same number of K blocks and a tile may be shared by neighbouring CTAs.
// Returns false past the last segment.
__device__ __forceinline__ bool prefill_segment(int i, int c, int G, int num_tiles, int KB, bool stream_k, int& tile,
                                                int& kb0, int& kb1) {
  if (!stream_k) {
    tile = c + i * G;
    kb0 = 0;
    kb1 = KB;
    return tile < num_tiles;
  }
  const long long U = static_cast<long long>(num_tiles) * KB;
  const long long u0 = U * c / G, u1 = U * (c + 1) / G;
  const long long us = i == 0 ? u0 : (u0 / KB + i) * KB;
  if (us >= u1) return false;
  tile = static_cast<int>(us / KB);
  kb0 = static_cast<int>(us - static_cast<long long>(tile) * KB);
  const long long ue = u1 < static_cast<long long>(tile + 1) * KB ? u1 : static_cast<long long>(tile + 1) * KB;
  kb1 = static_cast<int>(ue - static_cast<long long>(tile) * KB);
  return true;
}

// CTA whose stream-K range holds unit u (U units over G CTAs).
__device__ __forceinline__ int prefill_unit_owner(long long u, long long U, int G) {
  return static_cast<int>(((u + 1) * G - 1) / U);
}

// Weight box for (128-row block nb, K block kb) in either supported layout.
__device__ __forceinline__ void load_weight_box(void* dst, const CUtensorMap* map, uint64_t* bar, int nb, int kb,
                                                int KB, int tiled, uint64_t policy) {
  if (tiled)
    tma_load_2d(dst, map, bar, 0, (nb * KB + kb) * 128, policy);
  else
    tma_load_2d(dst, map, bar, kb * 128, nb * 128, policy);
}

// Pair form: the box's bytes are counted on the leader's barrier at shared::cluster address `bar`.
__device__ __forceinline__ void load_weight_box_pair(void* dst, const CUtensorMap* map, uint32_t bar, int nb, int kb,
                                                     int KB, int tiled, uint64_t policy) {
  if (tiled)
    tma_load_2d_pair(dst, map, bar, 0, (nb * KB + kb) * 128, policy);
  else
    tma_load_2d_pair(dst, map, bar, kb * 128, nb * 128, policy);
}

// Rows 64h .. 64h+63 of the weight box (nb, kb), through a map whose box is 64 rows high.
__device__ __forceinline__ void load_weight_half(void* dst, const CUtensorMap* map, uint64_t* bar, int nb, int h,
                                                 int kb, int KB, int tiled, uint64_t policy) {
  if (tiled)
    tma_load_2d(dst, map, bar, 0, (nb * KB + kb) * 128 + 64 * h, policy);
  else
    tma_load_2d(dst, map, bar, kb * 128, nb * 128 + 64 * h, policy);
}
__device__ __forceinline__ void load_weight_half_pair(void* dst, const CUtensorMap* map, uint32_t bar, int nb, int h,
                                                      int kb, int KB, int tiled, uint64_t policy) {
  if (tiled)
    tma_load_2d_pair(dst, map, bar, 0, (nb * KB + kb) * 128 + 64 * h, policy);
  else
    tma_load_2d_pair(dst, map, bar, kb * 128, nb * 128 + 64 * h, policy);
}

__device__ __forceinline__ void prefetch_weight_box(const CUtensorMap* map, int nb, int kb, int KB, int tiled) {
  if (tiled)
    tma_prefetch_l2_2d(map, 0, (nb * KB + kb) * 128);
  else
    tma_prefetch_l2_2d(map, kb * 128, nb * 128);
}

// SK (plain, one CTA per tile only): stream-K, CTAs take equal ranges of (tile, K block) units; the partial
// tiles go through p.ws with per-tile arrival counters in p.cnt.
template <bool FUSED, bool PAIR, bool SK = false>
__global__ void __launch_bounds__(PrefillCfg<FUSED, PAIR>::kThreads, 1)
    k_prefill(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const GemmParams p) {
  static_assert(!SK || (!FUSED && !PAIR), "stream-K runs the plain kernel on single CTAs");
  using Cfg = PrefillCfg<FUSED, PAIR>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* full = bars;              // [S]   TMA -> MMA
  uint64_t* empty = bars + S;         // [S]   MMA -> TMA
  uint64_t* pfull = bars + 2 * S;     // [2]   MMA -> promotion
  uint64_t* pempty = bars + 2 * S + 2;  // [2] promotion -> MMA
  uint64_t* drain = bars + 2 * S + 4;   // [1] MMA teardown
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);  // stream-K: this CTA finishes the tile
  float* xch = reinterpret_cast<float*>(smem + S * Cfg::kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Pair: rank 0 (leader) issues the MMAs for both CTAs; both CTAs' TMA loads count their bytes on
  // the leader's full barriers, and the peer hands TMEM buffers back on the leader's barriers.
  const uint32_t cr = PAIR ? cluster_ctarank() : 0u;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);  // the (leader's) producer's arrive.expect_tx
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], PAIR ? 256 + 8 : 256);  // own promotion threads (+ the peer's 8 warps)
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // the peer's barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) grid_dep_launch();

  const int M = p.M, KB = p.KB;
  const int nblk = p.N / 128;                       // 128-row weight blocks
  const int I_blk = FUSED ? nblk / 2 : 0;           // fused: gate blocks (= up blocks)
  const int num_m = (M + Cfg::kRows - 1) / Cfg::kRows;
  const int num_n = FUSED ? I_blk : (nblk + 1) / 2;
  const int num_tiles = num_m * num_n;
  const int tile0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tstep = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  constexpr bool sk = SK;
  const int row0 = PAIR ? static_cast<int>(cr) * 128 : 0;  // this CTA's first row inside a tile

  // Each role changes its register budget at the top of its own branch: code after a merge of
  // the two branches must fit the smaller budget, and only the short teardown follows one.
  if (warp >= 8) {
    regs_decrease<Cfg::Regs::kProducer>();
  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      grid_dep_wait();  // A and the output may belong to the previous kernel on the stream
      // The activation rows of a group are kept in L2 while the weight tiles pass.
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_normal();
      int s = 0;
      uint32_t ph = 0, issued = 0, parity_bits = 0;
      bool ok = true;
      BS_TR_DECL(1);
      int tile, kbs, kbe;
      for (int seg = 0; ok && prefill_segment(seg, tile0, tstep, num_tiles, KB, sk, tile, kbs, kbe); ++seg) {
        int tm, tn;
        prefill_tile_coords(tile, num_m, num_n, p.group_m, tm, tn);
        const int nb0 = FUSED ? tn : 2 * tn;
        const int nb1 = FUSED ? tn + I_blk : 2 * tn + 1;
        for (int kb = kbs; kb < kbe; ++kb) {
          BS_TR_MARK();
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          BS_TR_ADD(0);
          uint8_t* st = smem + s * Cfg::kStageBytes;
          if constexpr (PAIR) {
            // The leader expects both CTAs' bytes; the peer's loads may land before that, which only
            // takes the transaction count below zero until the leader's arrival.
            const uint32_t lead_full = mapa_shared(&full[s], 0);
            if (cr == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);
            tma_load_2d_pair(st, &tmA, lead_full, kb * 128, tm * Cfg::kRows + row0, pol_a);
            if constexpr (FUSED) {
              // weight rows [gate half cr | up half cr]: 64-row boxes
              load_weight_half_pair(st + Cfg::kABytes, &tmB, lead_full, nb0, cr, kb, KB, p.b_tiled, pol_b);
              load_weight_half_pair(st + Cfg::kABytes + 8192, &tmB, lead_full, nb1, cr, kb, KB, p.b_tiled, pol_b);
            } else {
              load_weight_box_pair(st + Cfg::kABytes, &tmB, lead_full, cr == 0 ? nb0 : nb1, kb, KB, p.b_tiled,
                                   pol_b);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
            tma_load_2d(st, &tmA, &full[s], kb * 128, tm * Cfg::kRows, pol_a);
            if constexpr (FUSED) {
              // weight rows [gate 0-63 | up 0-63 | gate 64-127 | up 64-127]: 64-row boxes
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                load_weight_half(st + Cfg::kABytes + 16384 * h, &tmB, &full[s], nb0, h, kb, KB, p.b_tiled, pol_b);
                load_weight_half(st + Cfg::kABytes + 16384 * h + 8192, &tmB, &full[s], nb1, h, kb, KB, p.b_tiled,
                                 pol_b);
              }
            } else {
              load_weight_box(st + Cfg::kABytes, &tmB, &full[s], nb0, kb, KB, p.b_tiled, pol_b);
              load_weight_box(st + Cfg::kABytes + 16384, &tmB, &full[s], nb1, kb, KB, p.b_tiled, pol_b);
            }
          }
          issued |= 1u << s;
          parity_bits = (parity_bits & ~(1u << s)) | (ph << s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      BS_TR_FLUSH(0, 1);
      if (!ok) {
        if constexpr (PAIR) {
          // The copies complete on the leader's barrier, which the peer cannot observe and which also
          // waits for the other CTA's bytes: give them time to land (they take microseconds).
          pause_ns(2000000ull);
        } else {
          // Leave no copy in flight: wait (bounded) for the last fill of every stage.
          for (int i = 0; i < S; ++i)
            if (issued & (1u << i))
              mbar_wait(&full[i], (parity_bits >> i) & 1u, abort_flag, p.status, kErrTimeoutDrain, 100000000ull);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && cr == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(Cfg::kRows, 256);
      int s = 0, b = 0;
      uint32_t ph = 0, pph = 0;
      bool ok = true;
      BS_TR_DECL(2);
      int tile, kbs, kbe;
      for (int seg = 0; ok && prefill_segment(seg, tile0, tstep, num_tiles, KB, sk, tile, kbs, kbe); ++seg) {
        for (int kb = kbs; kb < kbe; ++kb) {
          BS_TR_MARK();
          if (!mbar_wait(&full[s], ph, abort_flag, p.status, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          BS_TR_ADD(0);
          if (!mbar_wait(&pempty[b], pph ^ 1, abort_flag, p.status, kErrTimeoutPEmpty)) {
            ok = false;
            break;
          }
          BS_TR_ADD(1);
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t b0 = a0 + Cfg::kABytes;
          const uint32_t d = tmem + static_cast<uint32_t>(b * 256);
          if constexpr (PAIR) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_e4m3_pair(d, desc_kmajor_sw128(a0 + 32 * k), desc_kmajor_sw128(b0 + 32 * k), idesc,
                            k > 0 ? 1u : 0u);
            mma_commit_pair(&empty[s], 3);  // both CTAs' stage s is free again
            mma_commit_pair(&pfull[b], 3);  // both CTAs' partial buffer b is ready
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_e4m3(d, desc_kmajor_sw128(a0 + 32 * k), desc_kmajor_sw128(b0 + 32 * k), idesc, k > 0 ? 1u : 0u);
            mma_commit(&empty[s]);
            mma_commit(&pfull[b]);
          }
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
          if (++b == 2) {
            b = 0;
            pph ^= 1;
          }
        }
      }
      BS_TR_FLUSH(4, 2);
      // Every MMA issued so far completes before TMEM is released.
      if constexpr (PAIR)
        mma_commit_pair(drain, 1);
      else
        mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, p.status, kErrTimeoutDrain, 100000000ull);
    }
  }
  } else {
    regs_increase<Cfg::Regs::kConsumer>();
    grid_dep_wait();
    // ------------------------------------------------------------ promotion + epilogue
    // Plain: warpgroup wg owns TMEM columns 128wg..+127, i.e. weight block 2tn + wg, one scale per K block.
    // Fused: the MMA's 256 columns are [gate 0-63 | up 0-63 | gate 64-127 | up 64-127] of gate block tn and
    // up block tn + I/128, so warpgroup wg holds gate and up of the same 64 output columns 64wg..64wg+63
    // (accumulator pairs 0-31 gate, 32-63 up) and SiLU(g)*u needs no exchange: two scales per K block.
    const int wg = warp >> 2;
    const int q = warp & 3;           // TMEM lane quarter
    const int r = q * 32 + lane;      // row inside the tile
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t lead_pempty = PAIR ? mapa_shared(&pempty[0], 0) : 0u;  // the leader's pempty[0]
    // After an abort these warps keep walking the tile loop (skipping every wait, TMEM read and
    // store) so that both warpgroups still meet at the same named barriers.
    int b = 0;
    uint32_t pph = 0;
    bool ok = true;
    BS_TR_DECL(4);
    int tile, kbs, kbe;
    for (int seg = 0; prefill_segment(seg, tile0, tstep, num_tiles, KB, sk, tile, kbs, kbe); ++seg) {
      int tm, tn;
      prefill_tile_coords(tile, num_m, num_n, p.group_m, tm, tn);
      const int row = tm * Cfg::kRows + row0 + r;
      const bool row_ok = row < M;
      // plain: this warpgroup's weight block; fused: the gate block (the up block is I_blk further)
      const int nb = FUSED ? tn : 2 * tn + wg;
      const bool col_ok = nb < nblk;
      const float* as_row = p.As + static_cast<size_t>(row_ok ? row : 0) * KB;
      const float* bs_row = p.Bs + static_cast<size_t>(col_ok ? nb : 0) * KB;
      const float* bu_row = p.Bs + static_cast<size_t>(FUSED ? nb + I_blk : 0) * KB;

      uint64_t acc[64];  // column pairs (2i, 2i+1) of this thread's 128 columns
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0;

      // One K block: wait for its partial, fold it into the accumulators with the scale products sc2 (the
      // first 64 columns) and scu2 (the last 64), and hand the TMEM buffer back as soon as it is in registers.
      auto promote = [&](uint64_t sc2, uint64_t scu2) {
        if (ok && !mbar_wait(&pfull[b], pph, abort_flag, p.status, kErrTimeoutPFull)) ok = false;
        if (ok) {
          tc_fence_after();
          const uint32_t tbase = tmem + lane_addr + static_cast<uint32_t>(b * 256 + wg * 128);
          uint32_t v[64];
          tmem_ld64(tbase, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) ffma2(acc[i], v[2 * i], v[2 * i + 1], sc2);
          tmem_ld64(tbase + 64, v);
          tmem_ld_wait();
          // every column of the buffer this thread needs is in registers (the loads completed)
          if (!PAIR || cr == 0) {
            mbar_arrive(&pempty[b]);
          } else {
            // The leader's MMA reuses it: one relaxed arrival per warp on the leader's barrier (a
            // cluster-scope release arrival here costs a fence per K block on the critical path).
            __syncwarp();
            if (lane == 0) {
              tc_fence_before();
              mbar_arrive_remote_relaxed(lead_pempty + 8u * static_cast<uint32_t>(b));
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) ffma2(acc[32 + i], v[2 * i], v[2 * i + 1], scu2);
        }
        if (++b == 2) {
          b = 0;
          pph ^= 1;
        }
      };

      // Rows past M and the missing half of an odd last column tile read row 0 / block 0: their A rows and
      // weight rows are zero-filled by TMA, so the partial they scale is zero.
      if constexpr (FUSED) {
        // Scales in groups of four K blocks, one group ahead: the loads for K blocks kb0+4 .. kb0+7 are issued
        // when the group kb0 .. kb0+3 starts and handed over when it ends, so a load has four K blocks to land.
        // (Refilling each register right after reading it, with no hand-over, measured 20% slower.)
        constexpr int D = 4;
        float sa[D], sg[D], su[D];
#pragma unroll
        for (int j = 0; j < D; ++j) {
          const int k = j < KB ? j : KB - 1;
          sa[j] = ldg_f32(as_row + k);
          sg[j] = ldg_f32(bs_row + k);
          su[j] = ldg_f32(bu_row + k);
        }
        for (int kb0 = 0; kb0 < KB; kb0 += D) {
          float na[D], ng[D], nu[D];
#pragma unroll
          for (int j = 0; j < D; ++j) {
            const int kn = kb0 + D + j < KB ? kb0 + D + j : KB - 1;
            na[j] = ldg_f32(as_row + kn);
            ng[j] = ldg_f32(bs_row + kn);
            nu[j] = ldg_f32(bu_row + kn);
          }
#pragma unroll
          for (int j = 0; j < D; ++j) {
            if (kb0 + j >= KB) break;
            const float scg = __fmul_rn(sa[j], sg[j]), scu = __fmul_rn(sa[j], su[j]);
            promote(pack_f2(scg, scg), pack_f2(scu, scu));
          }
#pragma unroll
          for (int j = 0; j < D; ++j) {
            sa[j] = na[j];
            sg[j] = ng[j];
            su[j] = nu[j];
          }
        }
      } else {
        // Scales two K blocks ahead through a pair of registers (the deeper grouping above spills here).
        const int kn1 = kbs + 1 < kbe ? kbs + 1 : kbs;
        float a_n0 = ldg_f32(as_row + kbs), b_n0 = ldg_f32(bs_row + kbs);
        float a_n1 = ldg_f32(as_row + kn1), b_n1 = ldg_f32(bs_row + kn1);
        for (int kb = kbs; kb < kbe; ++kb) {
          const float sa = a_n0, sb = b_n0;
          a_n0 = a_n1;
          b_n0 = b_n1;
          if (kb + 2 < kbe) {
            a_n1 = ldg_f32(as_row + kb + 2);
            b_n1 = ldg_f32(bs_row + kb + 2);
          }
          const float sc = __fmul_rn(sa, sb);
          promote(pack_f2(sc, sc), pack_f2(sc, sc));
        }
      }

      if constexpr (SK) {
        if (!(kbs == 0 && kbe == KB)) {
          // Stream-K, a tile shared with other CTAs: store this CTA's partial (fp32, [slot][half][4-column group]
          // [row] as float4, so a warp's stores are contiguous), count the arrival, and let the last arriver add
          // every contributor's partial in CTA order and run the epilogue. Nobody waits on another CTA.
          const long long U = static_cast<long long>(num_tiles) * KB;
          const long long tu0 = static_cast<long long>(tile) * KB;
          const int c = static_cast<int>(blockIdx.x), G = static_cast<int>(gridDim.x);
          const int c_first = prefill_unit_owner(tu0, U, G), c_last = prefill_unit_owner(tu0 + KB - 1, U, G);
          const long long cu0 = U * c / G;
          const int my_slot = (c == c_first && cu0 < tu0) ? 1 : 0;
          float4* part = reinterpret_cast<float4*>(p.ws) + (static_cast<size_t>(c * 2 + my_slot) * 2 + wg) * 4096 + r;
          if (ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              part[j * 128] = make_float4(lo_f(acc[2 * j]), hi_f(acc[2 * j]), lo_f(acc[2 * j + 1]),
                                          hi_f(acc[2 * j + 1]));
          }
          // The barrier orders every promotion thread's stores before thread 0's counter increment, one acq_rel
          // atomic at device scope: its release (cumulative through the barrier) publishes the partials, its
          // acquire orders the finisher's reads below (after the next barrier).
          named_bar_sync(1, 256);
          if (threadIdx.x == 0) {
            int prev;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(p.cnt + tile) : "memory");
            const int last = prev == c_last - c_first;
            if (last) p.cnt[tile] = 0;
            *last_flag = last;
          }
          named_bar_sync(1, 256);
          // (thread 0 rewrites the flag only after the first barrier of a later shared segment, which every
          // thread reaches after this read)
          if (*last_flag == 0) continue;
#pragma unroll
          for (int i = 0; i < 64; ++i) acc[i] = 0;
          for (int cc = c_first; cc <= c_last; ++cc) {
            const int sl = (cc == c_first && U * cc / G < tu0) ? 1 : 0;
            const float4* src = reinterpret_cast<const float4*>(p.ws) + (static_cast<size_t>(cc * 2 + sl) * 2 + wg) * 4096 + r;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float4 v = __ldcg(src + j * 128);
              acc[2 * j] = pack_f2(lo_f(acc[2 * j]) + v.x, hi_f(acc[2 * j]) + v.y);
              acc[2 * j + 1] = pack_f2(lo_f(acc[2 * j + 1]) + v.z, hi_f(acc[2 * j + 1]) + v.w);
              if ((j & 15) == 15) compiler_fence();  // 16 loads in flight per thread
            }
          }
        }
      }

      BS_TR_MARK();
      if constexpr (!FUSED) {
        if (p.out_mc) {
          // Tensor-parallel partial added into every rank's output through the switch. Row-contiguous
          // runs travel best, so each warp transposes its 32 rows x 64 columns through a 4 KB buffer:
          // a thread writes its row's eight 16-byte chunks (XOR-swizzled by row), then each instruction
          // adds 4 rows x 128 contiguous bytes. col_ok is uniform per warp; every lane takes part.
          if (col_ok) {
            uint4* buf = reinterpret_cast<uint4*>(xch) + warp * 256;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const int j = 8 * h + c;  // columns 8j .. 8j+7 of this thread's 128
                buf[lane * 8 + (c ^ (lane & 7))] =
                    make_uint4(pack_bf16x2(lo_f(acc[4 * j]), hi_f(acc[4 * j])),
                               pack_bf16x2(lo_f(acc[4 * j + 1]), hi_f(acc[4 * j + 1])),
                               pack_bf16x2(lo_f(acc[4 * j + 2]), hi_f(acc[4 * j + 2])),
                               pack_bf16x2(lo_f(acc[4 * j + 3]), hi_f(acc[4 * j + 3])));
              }
              __syncwarp();
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int rr = 4 * i + (lane >> 3), cc = lane & 7;
                const int grow = tm * Cfg::kRows + row0 + q * 32 + rr;
                const uint4 v = buf[rr * 8 + (cc ^ (rr & 7))];
                if (ok && grow < M)
                  multimem_add_bf16x8(static_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(grow) * p.ldc +
                                          static_cast<size_t>(nb) * 128 + h * 64 + cc * 8,
                                      v);
              }
              __syncwarp();
            }
          }
        } else if (ok && row_ok && col_ok) {
          if (p.out_f32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<size_t>(row) * p.ldc +
                                                    static_cast<size_t>(nb) * 128);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              dst[j] = make_float4(lo_f(acc[2 * j]), hi_f(acc[2 * j]), lo_f(acc[2 * j + 1]), hi_f(acc[2 * j + 1]));
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) +
                                                  static_cast<size_t>(row) * p.ldc + static_cast<size_t>(nb) * 128);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              dst[j] = make_uint4(pack_bf16x2(lo_f(acc[4 * j]), hi_f(acc[4 * j])),
                                  pack_bf16x2(lo_f(acc[4 * j + 1]), hi_f(acc[4 * j + 1])),
                                  pack_bf16x2(lo_f(acc[4 * j + 2]), hi_f(acc[4 * j + 2])),
                                  pack_bf16x2(lo_f(acc[4 * j + 3]), hi_f(acc[4 * j + 3])));
          }
        }
      } else {
        // y = silu(g) * u for this thread's 64 columns (64wg .. 64wg+63 of the quant group), in place of the
        // gate accumulators; the 128-wide group's amax is the max of the two warpgroups' halves, met through
        // amax_x. scale = max(amax, 1e-10) / 448, inv = 1 / scale, q = sat_e4m3(y * inv) (H:532-579).
        float* amax_x = xch;  // [128 rows][2 halves]
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float y0 = silu_mul(lo_f(acc[i]), lo_f(acc[32 + i]));
          const float y1 = silu_mul(hi_f(acc[i]), hi_f(acc[32 + i]));
          acc[i] = pack_f2(y0, y1);
          amax = fmaxf(amax, fmaxf(fabsf(y0), fabsf(y1)));
        }
        amax_x[r * 2 + wg] = amax;
        named_bar_sync(1, 256);
        amax = fmaxf(amax_x[r * 2], amax_x[r * 2 + 1]);
        const float scale = __fdiv_rn(fmaxf(amax, 1e-10f), 448.0f);
        const float inv = __fdiv_rn(1.0f, scale);
        if (ok && row_ok) {
          const int I = I_blk * 128;
          if (wg == 0) p.qs[static_cast<size_t>(row) * I_blk + tn] = scale;
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + static_cast<size_t>(row) * I +
                                                static_cast<size_t>(tn) * 128 + wg * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const int e = 8 * j + 2 * h;  // pairs e, e+1: columns 16j + 4h .. +3 of this half
              w[h] = f2_to_e4m3x2(__fmul_rn(lo_f(acc[e]), inv), __fmul_rn(hi_f(acc[e]), inv)) |
                     (f2_to_e4m3x2(__fmul_rn(lo_f(acc[e + 1]), inv), __fmul_rn(hi_f(acc[e + 1]), inv)) << 16);
            }
            dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        named_bar_sync(1, 256);  // amax_x is free for the next tile
      }
      BS_TR_ADD(3);
    }
    if (lane == 0 && (warp & 3) == 0) BS_TR_FLUSH(8, 4);
  }

  // ------------------------------------------------------------ teardown
  // Multicast output: this thread's additions through the switch are complete before the kernel ends.
  if constexpr (!FUSED)
    if (p.out_mc && warp < 8) fence_acq_rel_sys();
  tc_fence_before();
  __syncthreads();
  // Pair: neither CTA leaves while the leader's MMAs (drained above) or the peer's remote
  // arrivals may still touch the other's shared memory or TMEM.
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, Cfg::kTmemCols);
    else
      tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace bs

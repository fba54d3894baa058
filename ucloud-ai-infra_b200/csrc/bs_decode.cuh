// Decode / speculative-verify block-scaled FP8 GEMM for sm_100a (M <= 128 tokens).
//
// Swap-AB: the weights are the MMA's M=128 operand and the tokens its N operand
// (N = NTP = M rounded up to 16), so one weight block of 128 rows x 128 K streams through the
// tensor core per K block and the tiny activation tile is re-read from L2. The promotion is the
// reference kernel's per-128-K-block arithmetic (patches/fp8_hand_sm89.py:189-199, :275-280)
// with the roles of rows and columns swapped:
//     acc[t] = fma(P_kb[row, t], As[t, kb] * Bs[nb, kb], acc[t])        (one thread per weight row)
//
// Work split ("stream-K"): a unit is one (weight tile, K block) pair; tile t covers units
// [t*KB, (t+1)*KB). CTA c of G takes the contiguous units [c*U/G, (c+1)*U/G), U = T*KB, so every
// SM streams the same number of weight bytes. A tile that straddles CTAs is finished by the
// CTA that arrives last on its counter: every contributor stores its fp32 partial in the
// workspace, and the last one sums them in CTA order (so the result does not depend on
// arrival order), resets the counter to zero and runs the epilogue. Nobody waits on another
// CTA, so no cross-CTA spin exists.
//
// CTA layout: NWG warpgroups of promotion warps (NWG = 1 plain, 2 fused: gate and up), then a
// warpgroup holding the TMA producer warp, the MMA/TMEM warp and two idle warps. The fused
// variant (384 threads) moves registers from that warpgroup to the promotion warps with
// setmaxnreg 40 / 232, as each promotion thread keeps NTP fp32 accumulators. TMEM holds two
// partial buffers of NWG*NTP columns.
//
// FUSED=true is the gate_up + SiLU*up + per-token-group quant front half at decode sizes: tile t
// is the pair (gate block t, up block t + I/128); the quant group of token tt is the 128 output
// columns of that pair, i.e. the 128 threads of the gate warpgroup, reduced through shared memory.
#pragma once
#include "bs_common.cuh"
#include "bs_prefill.cuh"

namespace bs {

__host__ __device__ constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

template <bool FUSED, int NTP>
struct DecodeCfg {
  static_assert(NTP % 16 == 0 && NTP >= 16 && NTP <= 128, "tokens per MMA must be 16..128, step 16");
  static constexpr int kNwg = FUSED ? 2 : 1;
  static constexpr int kPromo = 128 * kNwg;
  static constexpr int kThreads = kPromo + 128;
  static constexpr bool kSplitRegs = FUSED;  // 384 threads: registers move to the promotion warps
  using Regs = RegSplit<384, 168, 40, 232>;   // used when kSplitRegs
  static constexpr int kLaunchRegs = kSplitRegs ? Regs::kLaunch : 0;
  static constexpr int kWBytes = 16384 * kNwg;
  static constexpr int kXBytes = NTP * 128;
  static constexpr int kStageBytes = ((kWBytes + kXBytes + 1023) / 1024) * 1024;
  static constexpr int kXchBytes = FUSED ? NTP * 128 * 4 : 0;
  static constexpr int kRingBytes = 3 * kNwg * NTP * 4;
  static constexpr int kMaxSmem = 232448;  // 227 KB opt-in limit per block on sm_100
  static constexpr int kStagesRaw = (kMaxSmem - 1024 - kXchBytes - kRingBytes - 256) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static_assert(kStages >= 2, "decode pipeline needs two stages");
  static constexpr int kXchOff = kStages * kStageBytes;
  static constexpr int kRingOff = kXchOff + kXchBytes;
  static constexpr int kBarOff = kRingOff + kRingBytes;
  static constexpr int kSmemUsed = kBarOff + 256;
  // Ask for more than half of the SM's shared memory so a second CTA (and a second TMEM
  // allocation) can never land on the same SM.
  static constexpr int kSmemBytes = (kSmemUsed > 120 * 1024 ? kSmemUsed : 120 * 1024) + 1024;
  static constexpr int kTmemCols = pow2_at_least(2 * kNwg * NTP);
  static_assert(kTmemCols <= 512, "TMEM budget");
};

// Loads N consecutive TMEM columns (N a multiple of 16, at most 64) of this warp's 32 lanes into
// v[0..N) with every load in flight at once, then waits once.
template <int N>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, uint32_t (&v)[64]) {
  static_assert(N % 16 == 0 && N <= 64, "column group");
  if constexpr (N == 64) {
    tmem_ld64(taddr, v);
  } else {
#pragma unroll
    for (int c = 0; c + 32 <= N; c += 32) tmem_ld32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&v[c]));
    if constexpr (N % 32 == 16) tmem_ld16(taddr + (N - 16), *reinterpret_cast<uint32_t(*)[16]>(&v[N - 16]));
  }
  tmem_ld_wait();
}

// CTA that owns unit u when U units are split into G contiguous ranges [c*U/G, (c+1)*U/G).
__device__ __forceinline__ int unit_owner(long long u, long long U, int G) {
  return static_cast<int>(((u + 1) * G - 1) / U);
}

template <bool FUSED, int NTP>
__global__ void __launch_bounds__(DecodeCfg<FUSED, NTP>::kThreads, 1)
    k_decode(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
             const GemmParams p) {
  using Cfg = DecodeCfg<FUSED, NTP>;
  constexpr int S = Cfg::kStages;
  constexpr int NWG = Cfg::kNwg;
  constexpr int NPROMO = Cfg::kPromo;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* xch = reinterpret_cast<float*>(smem + Cfg::kXchOff);
  float* ring = reinterpret_cast<float*>(smem + Cfg::kRingOff);  // [3][NWG][NTP] scale products
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* pfull = bars + 2 * S;
  uint64_t* pempty = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int prod_warp = NPROMO / 32;
  const int mma_warp = prod_warp + 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], NPROMO / 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  if (warp == mma_warp) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int M = p.M, KB = p.KB;
  const int nblk = p.N / 128;
  const int I_blk = FUSED ? nblk / 2 : 0;
  const int T = FUSED ? I_blk : nblk;
  const long long U = static_cast<long long>(T) * KB;
  const int G = gridDim.x;
  const int c = blockIdx.x;
  const long long u0 = static_cast<long long>(c) * U / G;
  const long long u1 = static_cast<long long>(c + 1) * U / G;

  // Each role changes its register budget at the top of its own branch (see k_prefill).
  if (warp >= prod_warp) {
    if constexpr (Cfg::kSplitRegs) regs_decrease<Cfg::Regs::kProducer>();
  if (warp == prod_warp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      const uint64_t pol_w = policy_evict_first();  // weights stream through L2 once
      const uint64_t pol_x = policy_evict_last();   // activations are re-read by every CTA
      int s = 0;
      uint32_t ph = 0, issued = 0, parity_bits = 0;
      bool ok = true;
      BS_TR_DECL(1);
      for (long long u = u0; u < u1; ++u) {
        const int t = static_cast<int>(u / KB);
        const int kb = static_cast<int>(u - static_cast<long long>(t) * KB);
        BS_TR_MARK();
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        BS_TR_ADD(0);
        uint8_t* st = smem + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&full[s], Cfg::kWBytes + Cfg::kXBytes);
#pragma unroll
        for (int w = 0; w < NWG; ++w)
          load_weight_box(st + w * 16384, &tmW, &full[s], w == 0 ? t : t + I_blk, kb, KB, p.b_tiled, pol_w);
        tma_load_2d(st + Cfg::kWBytes, &tmX, &full[s], kb * 128, 0, pol_x);
        issued |= 1u << s;
        parity_bits = (parity_bits & ~(1u << s)) | (ph << s);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      BS_TR_FLUSH(0, 1);
      if (!ok) {
        for (int i = 0; i < S; ++i)
          if (issued & (1u << i))
            mbar_wait(&full[i], (parity_bits >> i) & 1u, abort_flag, p.status, kErrTimeoutDrain, 100000000ull);
      }
    }
  } else if (warp == mma_warp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, NTP);
      int s = 0, b = 0;
      uint32_t ph = 0, pph = 0;
      BS_TR_DECL(2);
      for (long long u = u0; u < u1; ++u) {
        BS_TR_MARK();
        if (!mbar_wait(&full[s], ph, abort_flag, p.status, kErrTimeoutFull)) break;
        BS_TR_ADD(0);
        if (!mbar_wait(&pempty[b], pph ^ 1, abort_flag, p.status, kErrTimeoutPEmpty)) break;
        BS_TR_ADD(1);
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * Cfg::kStageBytes);
        const uint32_t xs = st + Cfg::kWBytes;
#pragma unroll
        for (int w = 0; w < NWG; ++w) {
          const uint32_t d = tmem + static_cast<uint32_t>(b * NWG * NTP + w * NTP);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_e4m3(d, desc_kmajor_sw128(st + w * 16384 + 32 * k), desc_kmajor_sw128(xs + 32 * k), idesc,
                     k > 0 ? 1u : 0u);
        }
        mma_commit(&empty[s]);
        mma_commit(&pfull[b]);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
        if (++b == 2) {
          b = 0;
          pph ^= 1;
        }
      }
      BS_TR_FLUSH(4, 2);
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, p.status, kErrTimeoutDrain, 100000000ull);
    }
  }
  } else {
    if constexpr (Cfg::kSplitRegs) regs_increase<Cfg::Regs::kConsumer>();
    // ------------------------------------------------------------ promotion + epilogue
    // Every promotion thread runs the same sequence of named barriers whether or not the CTA
    // aborted; after an abort only the waits, TMEM reads and stores are skipped.
    const int tid = threadIdx.x;      // 0 .. NPROMO-1
    const int wg = warp >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;      // weight row inside the 128-row block
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;

    // Scale operands of unit u for token i: As[i, kb] and Bs[nb, kb]. The loads are issued from
    // always-valid addresses (last unit of the range, token 0 for padding tokens) and without a
    // select, because any instruction that consumed the result right away would wait for it.
    // The product and the padding mask are applied when the pair is stored to the shared ring,
    // two units later.
    const int ri = r < M ? r : 0;
    const bool r_live = r < M;
    struct ScalePair {
      float a, b;
    };
    auto load_scales = [&](long long u) -> ScalePair {
      const long long uc = u < u1 ? u : u1 - 1;
      const int t = static_cast<int>(uc / KB);
      const int kb = static_cast<int>(uc - static_cast<long long>(t) * KB);
      const int nb = wg == 0 ? t : t + I_blk;
      return {ldg_f32(p.As + static_cast<size_t>(ri) * KB + kb), ldg_f32(p.Bs + static_cast<size_t>(nb) * KB + kb)};
    };
    auto scale_value = [&](const ScalePair& s) -> float { return r_live ? __fmul_rn(s.a, s.b) : 0.f; };

    // Unit u's body stores the scale for u+1 (loaded two units earlier) into the ring and loads
    // the operands for u+3 into the registers it just freed. Two fixed register pairs alternate.
    if (r < NTP) ring[(0 * NWG + wg) * NTP + r] = (u0 < u1) ? scale_value(load_scales(u0)) : 0.f;
    ScalePair nxt_a = load_scales(u0 + 1);
    ScalePair nxt_b = load_scales(u0 + 2);
    named_bar_sync(1, NPROMO);

    uint64_t acc[NTP / 2];  // token pairs (2i, 2i+1)
#pragma unroll
    for (int i = 0; i < NTP / 2; ++i) acc[i] = 0;

    int b = 0;
    uint32_t pph = 0;
    bool ok = true;
    int slot = 0;                                   // ring slot of the current unit
    int seg_kb0 = static_cast<int>(u0 % KB);
    constexpr int G0 = NTP < 64 ? NTP : 64;         // first column group
    constexpr int G1 = NTP - G0;                    // second column group (NTP > 64)
    BS_TR_DECL(4);
    auto unit_body = [&](long long u, ScalePair& nxt) {
      const int t = static_cast<int>(u / KB);
      const int kb = static_cast<int>(u - static_cast<long long>(t) * KB);
      const int slot_next = slot == 2 ? 0 : slot + 1;
      BS_TR_MARK();
      if (r < NTP) ring[(slot_next * NWG + wg) * NTP + r] = scale_value(nxt);
      nxt = load_scales(u + 3);
      named_bar_sync(1, NPROMO);
      BS_TR_ADD(0);

      if (ok && !mbar_wait(&pfull[b], pph, abort_flag, p.status, kErrTimeoutPFull)) ok = false;
      BS_TR_ADD(1);
      if (ok) {
        tc_fence_after();
        const uint32_t tbase = tmem + lane_addr + static_cast<uint32_t>(b * NWG * NTP + wg * NTP);
        const ulonglong2* sc = reinterpret_cast<const ulonglong2*>(ring + (slot * NWG + wg) * NTP);
        uint32_t v[64];
        tmem_load_cols<G0>(tbase, v);
        if constexpr (G1 == 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[b]);
        }
#pragma unroll
        for (int i = 0; i < G0; i += 4) {
          const ulonglong2 s2 = sc[i / 4];
          ffma2(acc[i / 2], v[i], v[i + 1], s2.x);
          ffma2(acc[i / 2 + 1], v[i + 2], v[i + 3], s2.y);
        }
        if constexpr (G1 > 0) {
          tmem_load_cols<G1>(tbase + G0, v);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[b]);
#pragma unroll
          for (int i = 0; i < G1; i += 4) {
            const ulonglong2 s2 = sc[(G0 + i) / 4];
            ffma2(acc[(G0 + i) / 2], v[i], v[i + 1], s2.x);
            ffma2(acc[(G0 + i) / 2 + 1], v[i + 2], v[i + 3], s2.y);
          }
        }
      }
      BS_TR_ADD(2);
      if (++b == 2) {
        b = 0;
        pph ^= 1;
      }
      slot = slot_next;

      if (kb == KB - 1 || u + 1 == u1) {
        // ---------------- segment end: finish tile t (or hand over a partial)
        bool finisher = true;
        if (!(seg_kb0 == 0 && kb == KB - 1)) {
          const long long tu0 = static_cast<long long>(t) * KB;
          const int c_first = unit_owner(tu0, U, G);
          const int c_last = unit_owner(tu0 + KB - 1, U, G);
          const int my_slot = (c == c_first && u0 < tu0) ? 1 : 0;
          float* part = p.ws + (static_cast<size_t>(c * 2 + my_slot) * NWG + wg) * (NTP * 128) + r;
          if (ok) {
#pragma unroll
            for (int tt = 0; tt < NTP; ++tt)
              if (tt < M) part[tt * 128] = (tt & 1) ? hi_f(acc[tt / 2]) : lo_f(acc[tt / 2]);
          }
          __threadfence();
          named_bar_sync(1, NPROMO);
          if (tid == 0) {
            const int prev = atomicAdd(&p.cnt[t], 1);
            const int last = prev == c_last - c_first;
            if (last) p.cnt[t] = 0;
            *last_flag = last;
          }
          named_bar_sync(1, NPROMO);
          finisher = *last_flag != 0;
          if (finisher) {
            __threadfence();
#pragma unroll
            for (int i = 0; i < NTP / 2; ++i) acc[i] = 0;
            for (int cc = c_first; cc <= c_last; ++cc) {
              const int sl = (cc == c_first && (static_cast<long long>(cc) * U / G) < tu0) ? 1 : 0;
              const float* src = p.ws + (static_cast<size_t>(cc * 2 + sl) * NWG + wg) * (NTP * 128) + r;
#pragma unroll
              for (int tt = 0; tt < NTP; tt += 2) {
                const float x0 = tt < M ? __ldcg(src + tt * 128) : 0.f;
                const float x1 = tt + 1 < M ? __ldcg(src + (tt + 1) * 128) : 0.f;
                acc[tt / 2] = pack_f2(lo_f(acc[tt / 2]) + x0, hi_f(acc[tt / 2]) + x1);
                if ((tt & 15) == 14) compiler_fence();  // at most 16 loads in flight per thread
              }
            }
          }
        }
        if (finisher) {
          if constexpr (!FUSED) {
            if (ok) {
              const size_t col = static_cast<size_t>(t) * 128 + r;
              if (p.out_f32) {
                float* C = static_cast<float*>(p.out) + col;
#pragma unroll
                for (int tt = 0; tt < NTP; ++tt) {
                  if (tt < M) *C = (tt & 1) ? hi_f(acc[tt / 2]) : lo_f(acc[tt / 2]);
                  C += p.ldc;
                }
              } else {
                __nv_bfloat16* C = static_cast<__nv_bfloat16*>(p.out) + col;
#pragma unroll
                for (int tt = 0; tt < NTP; ++tt) {
                  if (tt < M) *C = __float2bfloat16_rn((tt & 1) ? hi_f(acc[tt / 2]) : lo_f(acc[tt / 2]));
                  C += p.ldc;
                }
              }
            }
          } else {
            // y = silu(g) * u, transposed to token-major in shared memory, then one pair of
            // threads per token quantises its 128-wide group.
            if (wg == 1) {
#pragma unroll
              for (int tt = 0; tt < NTP; ++tt) xch[tt * 128 + r] = (tt & 1) ? hi_f(acc[tt / 2]) : lo_f(acc[tt / 2]);
            }
            named_bar_sync(1, NPROMO);
            if (wg == 0) {
#pragma unroll
              for (int tt = 0; tt < NTP; ++tt)
                xch[tt * 128 + r] = silu_mul((tt & 1) ? hi_f(acc[tt / 2]) : lo_f(acc[tt / 2]), xch[tt * 128 + r]);
            }
            named_bar_sync(1, NPROMO);
            const int tok = tid >> 1;
            const int h = tid & 1;
            if (tok < NTP) {
              const float4* y4 = reinterpret_cast<const float4*>(xch + tok * 128 + h * 64);
              float y[64];
              float amax = 0.f;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float4 v = y4[i];
                y[4 * i] = v.x;
                y[4 * i + 1] = v.y;
                y[4 * i + 2] = v.z;
                y[4 * i + 3] = v.w;
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
              }
              amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
              const float scale = __fdiv_rn(fmaxf(amax, 1e-10f), 448.0f);
              const float inv = __fdiv_rn(1.0f, scale);
              if (ok && tok < M) {
                const int I = I_blk * 128;
                uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + static_cast<size_t>(tok) * I +
                                                      static_cast<size_t>(t) * 128 + h * 64);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  uint32_t w[4];
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    const int e = 16 * j + 4 * k;
                    w[k] = f2_to_e4m3x2(__fmul_rn(y[e], inv), __fmul_rn(y[e + 1], inv)) |
                           (f2_to_e4m3x2(__fmul_rn(y[e + 2], inv), __fmul_rn(y[e + 3], inv)) << 16);
                  }
                  dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
                }
                if (h == 0) p.qs[static_cast<size_t>(tok) * I_blk + t] = scale;
              }
            }
            named_bar_sync(1, NPROMO);
          }
        }
#pragma unroll
        for (int i = 0; i < NTP / 2; ++i) acc[i] = 0;
        seg_kb0 = 0;
        BS_TR_ADD(3);
      }
    };
    for (long long u = u0; u < u1; u += 2) {
      unit_body(u, nxt_a);
      if (u + 1 < u1) unit_body(u + 1, nxt_b);
    }
    if (lane == 0 && q == 0) BS_TR_FLUSH(8, 4);
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == mma_warp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace bs

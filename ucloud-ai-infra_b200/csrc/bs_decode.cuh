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
// CTA layout: PWG warpgroups of promotion warps, then one warpgroup with the TMA producer warp,
// the MMA/TMEM warp and one or two scale warps (two above 64 tokens). The MMA writes each unit's
// partial into one of up to four TMEM buffers of NWG*NTP columns (NWG = 1 plain, 2 fused: gate
// and up). The scale warps run ahead of the promotion and write each unit's scale products
// As[t,kb]*Bs[nb,kb] into a ring of eight slots in shared memory, so the promotion warps never
// wait on a global load and never synchronise with each other inside the K loop. Promotion
// warpgroup g owns the tokens [g*TR, (g+1)*TR) of every weight group (TR = NTP/PWG). Plain: one
// warpgroup up to 32 tokens, two at 48..64, four from 80. Fused: two warpgroups, four (each with gate and up of a
// quarter of the tokens) for 48..80 tokens. setmaxnreg moves registers from the producer
// warpgroup to the promotion warps (40/232 at 384 threads, 32/112 at 640).
//
// FUSED=true is the gate_up + SiLU*up + per-token-group quant front half at decode sizes: tile t
// is the pair (gate block t, up block t + I/128), both held by the same thread, so SiLU(g)*u needs
// no exchange. The quant group of token tt is the 128 weight rows of the tile, i.e. the four
// lane-quadrant warps of one promotion warpgroup: a warp-wide max, then a four-way max through
// shared memory. The quantised tile goes to shared memory in token-major rows and out with one
// TMA store.
#pragma once
#include <type_traits>

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
  static constexpr int kNwg = FUSED ? 2 : 1;               // weight blocks per unit: gate (+ up)
  // Promotion warpgroups. Fused at 96+ tokens: two warpgroups with 232 registers measured faster
  // than four with 112. Plain from 80 tokens: four warpgroups (20..32 tokens each) measured 4-8 % faster
  // than two (down_proj at 72..128 tokens, lm_head at 112 and 128, the config-1 GEMM); at 48..64 tokens
  // two stay faster.
  static constexpr int kPwg = FUSED ? (NTP >= 48 && NTP <= 80 ? 4 : 2) : (NTP >= 80 ? 4 : NTP >= 48 ? 2 : 1);
  static constexpr int kTr = NTP / kPwg;                   // tokens per promotion warpgroup
  static_assert(kTr % 4 == 0, "token range must be whole ulonglong2 scale loads");
  static constexpr int kPromo = 128 * kPwg;
  static constexpr int kThreads = kPromo + 128;
  static constexpr bool kSplitRegs = kPwg > 1;
  using Regs = typename std::conditional<kPwg == 4, RegSplit<640, 96, 32, 112>, RegSplit<384, 168, 40, 232>>::type;
  static constexpr int kLaunchRegs = kSplitRegs ? Regs::kLaunch : 0;
  static_assert(!kSplitRegs || Regs::kThreads == kThreads, "register split sized for this block");
  // Columns a promotion thread may hold from TMEM at once (registers left beside the accumulators).
  static constexpr int kLoadCols = kPwg == 4 ? 32 : 64;
  // Widest TMEM load issued at once when a unit's columns exceed kLoadCols.
  static constexpr int kChunk = kPwg == 4 ? 16 : 64;
  static constexpr int kWBytes = 16384 * kNwg;
  static constexpr int kXBytes = NTP * 128;
  static constexpr int kStageBytes = ((kWBytes + kXBytes + 1023) / 1024) * 1024;
  static constexpr int kBufCols = kNwg * NTP;               // TMEM columns of one partial buffer
  static constexpr int kBufs = 512 / kBufCols > 4 ? 4 : 512 / kBufCols;
  static constexpr int kTmemCols = pow2_at_least(kBufs * kBufCols);
  static_assert(kBufs >= 2 && kTmemCols <= 512, "TMEM budget");
  static constexpr int kSlots = 8;                          // scale-product ring depth, in units
  static constexpr int kScaleWarps = NTP > 64 ? 2 : 1;      // warps writing the scale products
  static constexpr int kRingBytes = kSlots * kNwg * NTP * 4;
  static constexpr int kAmaxBytes = FUSED ? 5 * NTP * 4 : 0;  // [4][NTP] warp maxima + [NTP] 1/scale
  static constexpr int kBarBytes = 512;
  static constexpr int kMaxSmem = 232448;  // 227 KB opt-in limit per block on sm_100
  static constexpr int kOutBytes = FUSED ? NTP * 128 : 0;    // token-major e4m3 rows of one tile
  static constexpr int kStagesRaw =
      (kMaxSmem - 1024 - kOutBytes - kRingBytes - kAmaxBytes - kBarBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static_assert(kStages >= 2, "decode pipeline needs two stages");
  static_assert((2 * kStages + 2 * kBufs + 2 * kSlots + 1) * 8 + 12 <= kBarBytes, "barrier area");
  static constexpr int kOutOff = kStages * kStageBytes;     // fused: quantised tile staged for TMA
  static constexpr int kRingOff = kOutOff + kOutBytes;
  static constexpr int kAmaxOff = kRingOff + kRingBytes;
  static constexpr int kBarOff = kAmaxOff + kAmaxBytes;
  static constexpr int kSmemUsed = kBarOff + kBarBytes;
  // Ask for more than half of the SM's shared memory so a second CTA (and a second TMEM
  // allocation) can never land on the same SM.
  static constexpr int kSmemBytes = (kSmemUsed > 120 * 1024 ? kSmemUsed : 120 * 1024) + 1024;
};

// CTA that owns unit u when U units are split into G contiguous ranges [c*U/G, (c+1)*U/G).
__device__ __forceinline__ int unit_owner(int u, int U, int G) {
  return ((u + 1) * G - 1) / U;
}

__device__ __forceinline__ float pair_elem(uint64_t v, int odd) { return odd ? hi_f(v) : lo_f(v); }

template <bool FUSED, int NTP>
__global__ void __launch_bounds__(DecodeCfg<FUSED, NTP>::kThreads, 1)
    k_decode(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
             const __grid_constant__ CUtensorMap tmO, const GemmParams p) {
  using Cfg = DecodeCfg<FUSED, NTP>;
  constexpr int S = Cfg::kStages;
  constexpr int NWG = Cfg::kNwg;
  constexpr int NB = Cfg::kBufs;
  constexpr int NS = Cfg::kSlots;
  constexpr int TR = Cfg::kTr;
  constexpr int NPROMO = Cfg::kPromo;
  constexpr int NPW = NPROMO / 32;  // promotion warps
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* ring = reinterpret_cast<float*>(smem + Cfg::kRingOff);  // [NS][NWG][NTP] scale products
  float* amx = reinterpret_cast<float*>(smem + Cfg::kAmaxOff);   // fused: [4][NTP] maxima, [NTP] 1/scale
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* pfull = empty + S;
  uint64_t* pempty = pfull + NB;
  uint64_t* sfull = pempty + NB;
  uint64_t* sempty = sfull + NS;
  uint64_t* drain = sempty + NS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int prod_warp = NPW;
  constexpr int mma_warp = NPW + 1;
  constexpr int scale_warp = NPW + 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], NPROMO);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&sfull[i], 32 * Cfg::kScaleWarps);
      mbar_init(&sempty[i], NPROMO);
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
  if (threadIdx.x == 0) grid_dep_launch();

  const int M = p.M, KB = p.KB;
  const int nblk = p.N / 128;
  const int I_blk = FUSED ? nblk / 2 : 0;
  const int T = FUSED ? I_blk : nblk;
  const int U = T * KB;  // the host keeps U * G below 2^31
  const int G = gridDim.x;
  const int c = blockIdx.x;
  const int u0 = static_cast<int>(static_cast<long long>(c) * U / G);
  const int u1 = static_cast<int>(static_cast<long long>(c + 1) * U / G);
  const int t0 = u0 / KB;       // tile and K block of the first unit; every loop steps both
  const int kb0 = u0 - t0 * KB;

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
      // The first stages' weights go to L2 while an earlier kernel may still be running.
      for (int u = u0, t = t0, kb = kb0; u < u1 && u < u0 + S; ++u, kb = kb + 1 == KB ? 0 : kb + 1, t += kb == 0)
#pragma unroll
        for (int w = 0; w < NWG; ++w) prefetch_weight_box(&tmW, w == 0 ? t : t + I_blk, kb, KB, p.b_tiled);
      grid_dep_wait();
      BS_TR_DECL(1);
      for (int u = u0, t = t0, kb = kb0; u < u1; ++u, kb = kb + 1 == KB ? 0 : kb + 1, t += kb == 0) {
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
      for (int u = u0; u < u1; ++u) {
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
          const uint32_t d = tmem + static_cast<uint32_t>(b * Cfg::kBufCols + w * NTP);
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
        if (++b == NB) {
          b = 0;
          pph ^= 1;
        }
      }
      BS_TR_FLUSH(4, 2);
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, p.status, kErrTimeoutDrain, 100000000ull);
    }
  } else if (warp < scale_warp + Cfg::kScaleWarps) {
    // ------------------------------------------------------------ scale products
    // Scale warp sw, lane l writes As[tok, kb] * Bs[nb_w, kb] for tokens
    // tok = sw*32*TPL + l + 32*j of unit u into ring slot u % NS (0 for padding tokens). The
    // operands of unit u+2 are loaded into the registers unit u has just used, from always-valid
    // addresses (the range's last unit, row 0 for padding tokens), so no store ever waits on a
    // load issued less than two units earlier.
    grid_dep_wait();
    constexpr int TPL = (NTP + 32 * Cfg::kScaleWarps - 1) / (32 * Cfg::kScaleWarps);
    const int tok_base = (warp - scale_warp) * 32 * TPL + lane;
    struct Ops {
      float a[TPL];
      float b[NWG];
    };
    int lu = u0, lt = t0, lkb = kb0;  // load cursor: the unit whose operands load next
    auto load_next = [&](Ops& o) {
#pragma unroll
      for (int j = 0; j < TPL; ++j) {
        const int tok = tok_base + 32 * j;
        o.a[j] = ldg_f32(p.As + ((tok < M ? tok : 0) * KB + lkb));
      }
#pragma unroll
      for (int w = 0; w < NWG; ++w) o.b[w] = ldg_f32(p.Bs + ((w == 0 ? lt : lt + I_blk) * KB + lkb));
      if (lu + 1 < u1) {  // stays on the last unit of the range once there
        ++lu;
        if (++lkb == KB) {
          lkb = 0;
          ++lt;
        }
      }
    };
    int slot = 0;
    uint32_t sph = 0;
    bool ok = true;
    BS_TR_DECL(1);
    auto body = [&](Ops& o) {
      BS_TR_MARK();
      if (!mbar_wait(&sempty[slot], sph ^ 1, abort_flag, p.status, kErrTimeoutPEmpty)) {
        ok = false;
        return;
      }
      BS_TR_ADD(0);
      float* dst = ring + slot * (NWG * NTP);
#pragma unroll
      for (int w = 0; w < NWG; ++w)
#pragma unroll
        for (int j = 0; j < TPL; ++j) {
          const int tok = tok_base + 32 * j;
          if (tok < NTP) dst[w * NTP + tok] = tok < M ? __fmul_rn(o.a[j], o.b[w]) : 0.f;
        }
      mbar_arrive(&sfull[slot]);
      load_next(o);
      if (++slot == NS) {
        slot = 0;
        sph ^= 1;
      }
    };
    Ops oa, ob;
    load_next(oa);
    load_next(ob);
    for (int u = u0; u < u1 && ok; u += 2) {
      body(oa);
      if (u + 1 < u1 && ok) body(ob);
    }
    if (lane == 0 && warp == scale_warp) BS_TR_FLUSH(16, 1);
  }
  } else {
    if constexpr (Cfg::kSplitRegs) regs_increase<Cfg::Regs::kConsumer>();
    grid_dep_wait();
    // ------------------------------------------------------------ promotion + epilogue
    // Every promotion thread runs the same sequence of named barriers whether or not the CTA
    // aborted; after an abort only the waits, TMEM reads and stores are skipped.
    const int tid = threadIdx.x;      // 0 .. NPROMO-1
    const int q = warp & 3;           // TMEM lane quadrant
    const int tok0 = (warp >> 2) * TR;
    const int r = q * 32 + lane;      // weight row inside the 128-row block
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;

    uint64_t acc[NWG][TR / 2];  // token pairs (tok0 + 2i, tok0 + 2i + 1) of each weight group
#pragma unroll
    for (int w = 0; w < NWG; ++w)
#pragma unroll
      for (int i = 0; i < TR / 2; ++i) acc[w][i] = 0;

    int b = 0, slot = 0;
    uint32_t pph = 0, sph = 0;
    bool ok = true;
    int seg_kb0 = kb0;
    BS_TR_DECL(4);
    for (int u = u0, t = t0, kb = kb0; u < u1; ++u, kb = kb + 1 == KB ? 0 : kb + 1, t += kb == 0) {
      BS_TR_MARK();
      if (ok && !mbar_wait(&pfull[b], pph, abort_flag, p.status, kErrTimeoutPFull)) ok = false;
      BS_TR_ADD(0);
      if (ok && !mbar_wait(&sfull[slot], sph, abort_flag, p.status, kErrTimeoutPFull)) ok = false;
      BS_TR_ADD(1);
      if (ok) {
        tc_fence_after();
        const uint32_t tb = tmem + lane_addr + static_cast<uint32_t>(b * Cfg::kBufCols + tok0);
        const ulonglong2* sc = reinterpret_cast<const ulonglong2*>(ring + slot * (NWG * NTP) + tok0);
        if constexpr (NWG * TR <= Cfg::kLoadCols) {
          // every column of the unit in flight at once, one wait
          uint32_t v[NWG * TR];
#pragma unroll
          for (int w = 0; w < NWG; ++w) tmem_ld_run<TR>(tb + w * NTP, v + w * TR);
          tmem_ld_wait();
          mbar_arrive(&pempty[b]);  // this thread's columns are in registers
#pragma unroll
          for (int w = 0; w < NWG; ++w)
#pragma unroll
            for (int i = 0; i < TR; i += 4) {
              const ulonglong2 s2 = sc[(w * NTP + i) / 4];
              ffma2(acc[w][i / 2], v[w * TR + i], v[w * TR + i + 1], s2.x);
              ffma2(acc[w][i / 2 + 1], v[w * TR + i + 2], v[w * TR + i + 3], s2.y);
            }
        } else {
          // one chunk of at most kChunk columns of one weight group at a time
          constexpr int CH = Cfg::kChunk;
#pragma unroll
          for (int w = 0; w < NWG; ++w) {
#pragma unroll
            for (int c0 = 0; c0 < TR; c0 += CH) {
              constexpr int kLast = TR - (TR - 1) / CH * CH;  // width of the final chunk
              uint32_t v[CH];
              if (c0 + CH <= TR)
                tmem_ld_run<CH>(tb + w * NTP + c0, v);
              else
                tmem_ld_run<kLast>(tb + w * NTP + c0, v);
              tmem_ld_wait();
              if (w == NWG - 1 && c0 + CH >= TR) mbar_arrive(&pempty[b]);
#pragma unroll
              for (int i = 0; i < CH; i += 4) {
                if (c0 + i < TR) {
                  const ulonglong2 s2 = sc[(w * NTP + c0 + i) / 4];
                  ffma2(acc[w][(c0 + i) / 2], v[i], v[i + 1], s2.x);
                  ffma2(acc[w][(c0 + i) / 2 + 1], v[i + 2], v[i + 3], s2.y);
                }
              }
            }
          }
        }
        mbar_arrive(&sempty[slot]);  // this thread's reads of the slot are done
      }
      BS_TR_ADD(2);
      if (++b == NB) {
        b = 0;
        pph ^= 1;
      }
      if (++slot == NS) {
        slot = 0;
        sph ^= 1;
      }

      if (kb == KB - 1 || u + 1 == u1) {
        // ---------------- segment end: finish tile t (or hand over a partial)
        bool finisher = true;
        if (!(seg_kb0 == 0 && kb == KB - 1)) {
          const int tu0 = t * KB;
          const int c_first = unit_owner(tu0, U, G);
          const int c_last = unit_owner(tu0 + KB - 1, U, G);
          const int my_slot = (c == c_first && u0 < tu0) ? 1 : 0;
          float* part = p.ws + static_cast<size_t>(c * 2 + my_slot) * NWG * (NTP * 128) + r;
          if (ok) {
#pragma unroll
            for (int w = 0; w < NWG; ++w)
#pragma unroll
              for (int i = 0; i < TR; ++i)
                if (tok0 + i < M) part[(w * NTP + tok0 + i) * 128] = pair_elem(acc[w][i / 2], i & 1);
          }
          // The barrier orders every promotion thread's partial stores before thread 0's counter increment, one
          // acq_rel atomic at device scope: its release (cumulative through the barrier) publishes the partials,
          // its acquire orders the finisher's reads below (after the next barrier).
          named_bar_sync(1, NPROMO);
          if (tid == 0) {
            int prev;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(p.cnt + t) : "memory");
            const int last = prev == c_last - c_first;
            if (last) p.cnt[t] = 0;
            *last_flag = last;
          }
          named_bar_sync(1, NPROMO);
          finisher = *last_flag != 0;
          if (finisher) {
#pragma unroll
            for (int w = 0; w < NWG; ++w)
#pragma unroll
              for (int i = 0; i < TR / 2; ++i) acc[w][i] = 0;
            for (int cc = c_first; cc <= c_last; ++cc) {
              const int sl = (cc == c_first && static_cast<int>(static_cast<long long>(cc) * U / G) < tu0) ? 1 : 0;
              const float* src = p.ws + static_cast<size_t>(cc * 2 + sl) * NWG * (NTP * 128) + r;
#pragma unroll
              for (int w = 0; w < NWG; ++w)
#pragma unroll
                for (int i = 0; i < TR; i += 2) {
                  const int tt = tok0 + i;
                  const float x0 = tt < M ? __ldcg(src + (w * NTP + tt) * 128) : 0.f;
                  const float x1 = tt + 1 < M ? __ldcg(src + (w * NTP + tt + 1) * 128) : 0.f;
                  acc[w][i / 2] = pack_f2(lo_f(acc[w][i / 2]) + x0, hi_f(acc[w][i / 2]) + x1);
                  if ((i & 15) == 14) compiler_fence();  // at most 16 loads in flight per thread
                }
            }
          }
        }
        if (finisher) {
          if constexpr (!FUSED) {
            const size_t col = static_cast<size_t>(t) * 128 + r;
            if (p.out_mc) {
              // Tensor-parallel partial added into every rank's output through the switch. The reduction
              // is 4 bytes wide, so an even row r sends the column pair (r, r + 1); lane r + 1 of the same
              // warp holds r + 1. Every lane takes part in the shuffle, whatever its `ok`.
              __nv_bfloat16* C = static_cast<__nv_bfloat16*>(p.out) + col;
#pragma unroll
              for (int i = 0; i < TR; ++i) {
                const float v = pair_elem(acc[0][i / 2], i & 1);
                const float nxt = __shfl_down_sync(0xffffffffu, v, 1);
                if (ok && tok0 + i < M && (r & 1) == 0)
                  multimem_add_bf16x2(C + static_cast<size_t>(tok0 + i) * p.ldc, pack_bf16x2(v, nxt));
              }
              fence_acq_rel_sys();
            } else if (ok) {
              if (p.out_f32) {
                float* C = static_cast<float*>(p.out) + col;
#pragma unroll
                for (int i = 0; i < TR; ++i)
                  if (tok0 + i < M) C[static_cast<size_t>(tok0 + i) * p.ldc] = pair_elem(acc[0][i / 2], i & 1);
              } else {
                __nv_bfloat16* C = static_cast<__nv_bfloat16*>(p.out) + col;
#pragma unroll
                for (int i = 0; i < TR; ++i)
                  if (tok0 + i < M)
                    C[static_cast<size_t>(tok0 + i) * p.ldc] = __float2bfloat16_rn(pair_elem(acc[0][i / 2], i & 1));
              }
            }
          } else {
            // y = silu(g) * u at weight row r for this warpgroup's tokens, in place of the gate
            // accumulators. The group max of |y| over the tile's 128 rows: a warp max (|y| orders
            // like its bit pattern), then a four-way max over the lane-quadrant warps through
            // shared memory. The reference's scale arithmetic (H:561, :577-578):
            // scale = max(amax, 1e-10) / 448, q = e4m3(y * (1 / scale)). The quantised tile is
            // transposed to token-major rows in shared memory and written by one TMA store.
            uint32_t m[TR];
#pragma unroll
            for (int i = 0; i < TR; i += 2) {
              const float y0 = silu_mul(lo_f(acc[0][i / 2]), lo_f(acc[1][i / 2]));
              const float y1 = silu_mul(hi_f(acc[0][i / 2]), hi_f(acc[1][i / 2]));
              acc[0][i / 2] = pack_f2(y0, y1);
              m[i] = __float_as_uint(fabsf(y0));
              m[i + 1] = __float_as_uint(fabsf(y1));
            }
            warp_max_halving<TR, 16>(m, lane);
            if ((lane & warp_max_dup_mask<TR, 16>()) == 0) {
              const int base = tok0 + warp_max_base<TR, 16>(lane);
#pragma unroll
              for (int i = 0; i < warp_max_count<TR, 16>(); ++i) amx[q * NTP + base + i] = __uint_as_float(m[i]);
            }
            named_bar_sync(1, NPROMO);
            if (tid < NTP) {
              const float am = fmaxf(fmaxf(amx[tid], amx[NTP + tid]), fmaxf(amx[2 * NTP + tid], amx[3 * NTP + tid]));
              const float scale = __fdiv_rn(fmaxf(am, 1e-10f), 448.0f);
              amx[4 * NTP + tid] = __fdiv_rn(1.0f, scale);
              if (ok && tid < M) p.qs[static_cast<size_t>(tid) * I_blk + t] = scale;
            }
            named_bar_sync(1, NPROMO);
            if (ok) {
              uint8_t* stg = smem + Cfg::kOutOff + r;
#pragma unroll
              for (int i = 0; i < TR; ++i)
                stg[(tok0 + i) * 128] = static_cast<uint8_t>(
                    f2_to_e4m3x2(__fmul_rn(pair_elem(acc[0][i / 2], i & 1), amx[4 * NTP + tok0 + i]), 0.f) & 0xffu);
              fence_proxy_async_smem();
            }
            named_bar_sync(1, NPROMO);
            if (ok && tid == 0) {
              tma_store_2d(&tmO, smem + Cfg::kOutOff, t * 128, 0);
              bulk_commit();
              bulk_wait_read_all();  // the staging rows are free again once read
            }
            named_bar_sync(1, NPROMO);
          }
        }
#pragma unroll
        for (int w = 0; w < NWG; ++w)
#pragma unroll
          for (int i = 0; i < TR / 2; ++i) acc[w][i] = 0;
        seg_kb0 = 0;
        BS_TR_ADD(3);
      }
    }
    if (lane == 0 && q == 0 && warp < 4) BS_TR_FLUSH(8, 4);
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

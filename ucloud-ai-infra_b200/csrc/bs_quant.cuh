// HBM-bound byte kernels of the path: per-token-group activation quant and the tile-first
// weight pre-pack.
#pragma once
#include "bs_common.cuh"

namespace bs {

constexpr int kQuantThreads = 256;

// Correctly rounded fp32 quotient x / s from r = RN(1/s): q0 = RN(x * r), e = x - s * q0 (exact in one
// fma), q = RN(q0 + e * r). This is Markstein's correction step (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; the quotient theorem in
// Muller et al., Handbook of Floating-Point Arithmetic, ch. 4): with r the correctly rounded reciprocal and
// q0 within one ulp of x / s, the remainder e is exact and q is RN(x / s), as long as no intermediate is
// subnormal. Here s >= 1e-12 and the only quotients that reach e4m3 above zero satisfy |x| >= 2^-10 * s,
// so the e4m3 byte always equals that of the IEEE quotient; the sign is copied from x so that x = -0
// gives -0. One reciprocal per 128-group replaces 128 IEEE divisions.
__device__ __forceinline__ float div_by_scale(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-s, q0, x);
  return copysignf(__fmaf_rn(e, r, q0), x);
}

// x bf16 [M, K] -> A e4m3 [M, K], As fp32 [M, K/128].
// Sixteen threads own one 128-wide group (8 elements = one 16-byte load each), reduce |x| with
// shuffles inside the half-warp, then
//     As = max(amax / 448, 1e-12),  A = e4m3_rn(x / As)
// which is the reference's torch quantiser (scripts/fp8_gemm_factor_check.py:22-27:
// `s = amax / FP8_MAX; s = s.clamp_min(1e-12); (x / s).to(float8_e4m3fn)`), computed in fp32
// with correctly rounded division (div_by_scale) so the bytes match it exactly. |x / As| <= 448 * (1 + 2^-23),
// which rounds to 448 under both torch's conversion and the saturating cvt used here.
__global__ void __launch_bounds__(kQuantThreads)
    k_group_quant(const __nv_bfloat16* __restrict__ x, int ldx, uint8_t* __restrict__ A, float* __restrict__ As,
                  int M, int K) {
  if (threadIdx.x == 0) grid_dep_launch();
  grid_dep_wait();  // x may be the previous kernel's output
  const int KB = K / 128;
  const long long groups = static_cast<long long>(M) * KB;
  const int sub = threadIdx.x & 15;
  // The loop bound is uniform per warp (two groups per warp per step) so that both half-warps
  // always take part in the full-mask shuffles; a half without a group only skips its memory ops.
  const long long warp_id = (static_cast<long long>(blockIdx.x) * kQuantThreads + threadIdx.x) >> 5;
  const long long step = static_cast<long long>(gridDim.x) * (kQuantThreads / 32) * 2;
  for (long long g2 = warp_id * 2; g2 < groups; g2 += step) {
    const long long g = g2 + ((threadIdx.x >> 4) & 1);
    const bool active = g < groups;
    const long long row = active ? g / KB : 0;
    const int kb = active ? static_cast<int>(g - row * KB) : 0;
    float v[8];
    if (active) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + row * ldx + kb * 128 + sub * 8));
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = fmaxf(__fdiv_rn(amax, 448.0f), 1e-12f);
    const float rs = __frcp_rn(s);
    if (active) {
      uint2 q;
      q.x = f2_to_e4m3x2(div_by_scale(v[0], s, rs), div_by_scale(v[1], s, rs)) |
            (f2_to_e4m3x2(div_by_scale(v[2], s, rs), div_by_scale(v[3], s, rs)) << 16);
      q.y = f2_to_e4m3x2(div_by_scale(v[4], s, rs), div_by_scale(v[5], s, rs)) |
            (f2_to_e4m3x2(div_by_scale(v[6], s, rs), div_by_scale(v[7], s, rs)) << 16);
      *reinterpret_cast<uint2*>(A + row * K + kb * 128 + sub * 8) = q;
      if (sub == 0) As[row * KB + kb] = s;
    }
  }
}

constexpr int kNormThreads = 256;  // eight warps per CTA
constexpr int kNormMaxK = 16384;

__device__ __forceinline__ void unpack_bf16x8(const uint4& raw, float (&v)[8]) {
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h2[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): each lane is one ordinary IEEE operation, rounded to nearest.
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t ffma2r(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// Two bf16 (low half = first element) -> the fp32 pair (exact: a bf16 is the top half of an fp32).
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t v) {
  return static_cast<uint64_t>(v << 16) | (static_cast<uint64_t>(v & 0xffff0000u) << 32);
}
// The group scale max(amax / 448, 1e-12), with amax / 448 correctly rounded by the same correction step
// from the correctly rounded reciprocal of 448 (a compile-time constant).
__device__ __forceinline__ float group_scale(float amax) {
  constexpr float kInv448 = 1.0f / 448.0f;
  const float q0 = __fmul_rn(amax, kInv448);
  return fmaxf(__fmaf_rn(__fmaf_rn(-448.0f, q0, amax), kInv448, q0), 1e-12f);
}

// -div_by_scale(y, s, r) on a pair, from neg_r = -r: nq0 = RN(y * -r) = -RN(y * r); e = RN(y + s * nq0), the
// same value and sign as div_by_scale's e; nq = RN(e * -r + nq0), whose addends are the negations of
// div_by_scale's. So nq = -div_by_scale(y) bit for bit, signed zeros included (y = -0 gives nq = +0): the
// e4m3 byte of the quotient is the byte of nq with its sign bit flipped, and no copysign is needed.
__device__ __forceinline__ uint64_t neg_div_by_scale2(uint64_t y, uint64_t s, uint64_t neg_r) {
  const uint64_t nq0 = fmul2(y, neg_r);
  return ffma2r(ffma2r(s, nq0, y), neg_r, nq0);
}

// Per half: max(|a|, |b|) of two packed bf16 pairs (the result's sign bits are the xor of the inputs' and are
// ignored by the caller). Exact: a comparison, no rounding.
__device__ __forceinline__ uint32_t bf16x2_absmax(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Per-token-group quant of rows, optionally after RMSNorm, in one HBM pass. A CTA of 256 threads owns one row
// at a time and walks rows blockIdx.x, blockIdx.x + gridDim.x, ...; thread t holds the row's 16-byte chunks
// c = t + 256 j (j < C), so each 128-group is the 16 chunks of one half-warp at one j. The loads of the next
// row are issued before the current row is processed, so the HBM stream does not stop for the row's
// reduction. NORM = false quantises x itself (the activation quant ahead of a linear); NORM = true has the
// rounding points of the unfused pair "RMSNorm -> per_token_group_quant_fp8":
//   h   = x                                   (or bf16_rn(x + residual) with RES, written back to residual)
//   ss  = sum of h*h in fp32 (products rounded, no fused multiply-add) in a fixed order that depends on K only:
//         thread t keeps two partial sums, of the even and of the odd elements of its chunks, adding
//         h[8c + 2e]^2 (resp. h[8c + 2e + 1]^2) for its chunks in increasing c and e = 0..3; its total is
//         even + odd; each warp combines its lanes in a butterfly (xor 16, 8, 4, 2, 1); the row's sum is the
//         eight warp totals added in warp order, ((w0 + w1) + w2) + ... + w7
//   rs  = 1 / sqrt(ss / K + eps)              (IEEE divide and square root)
//   y   = bf16_rn((h * rs) * w)               (the bf16 value an unfused RMSNorm stores)
// and then, in both cases,
//   As  = max(amax(y over 128) / 448, 1e-12),  A = e4m3_rn(y / As)   (the reference's torch quantiser,
//         scripts/fp8_gemm_factor_check.py:22-27, with correctly rounded division, div_by_scale)
// The arithmetic runs on fp32 pairs.
// CTAs per SM the register budget is sized for, per form (measured: the plain quant streams fastest at four,
// RMSNorm at three, RMSNorm with the residual at two).
template <bool NORM, bool RES>
constexpr int kRowMinCtas = NORM ? (RES ? 2 : 3) : 4;

template <int C, bool NORM, bool RES>
__global__ void __launch_bounds__(kNormThreads, kRowMinCtas<NORM, RES>)
    k_row_group_quant(const __nv_bfloat16* __restrict__ x, int ldx, __nv_bfloat16* residual, int ldr,
                      const __nv_bfloat16* __restrict__ w, float eps, uint8_t* __restrict__ A,
                      float* __restrict__ As, int M, int K) {
  static_assert(NORM || !RES, "the residual add belongs to the norm");
  constexpr int T = kNormThreads;
  __shared__ float warp_ss[2][T / 32];  // by row parity, so one barrier per row suffices
  if (threadIdx.x == 0) grid_dep_launch();
  grid_dep_wait();  // x and the residual may be the previous kernel's output
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t = threadIdx.x;
  const int nch = K / 8;
  const int KB = K / 128;

  auto load_row = [&](int row, uint4 (&xv)[C], uint4 (&rv)[C]) {
    const __nv_bfloat16* xr = x + static_cast<size_t>(row) * ldx;
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const int c = t + T * j;
      if (c < nch) xv[j] = __ldg(reinterpret_cast<const uint4*>(xr + c * 8));
    }
    if constexpr (RES) {
      const __nv_bfloat16* rr = residual + static_cast<size_t>(row) * ldr;
#pragma unroll
      for (int j = 0; j < C; ++j) {
        const int c = t + T * j;
        if (c < nch) rv[j] = *reinterpret_cast<const uint4*>(rr + c * 8);
      }
    }
  };

  // the norm weight's chunks of this thread, widened once for every row the CTA walks
  uint64_t wf[NORM ? C : 1][4];
  if constexpr (NORM) {
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const int c = t + T * j;
      if (c < nch) {
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + c * 8));
        const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
        for (int e = 0; e < 4; ++e) wf[j][e] = bf16x2_to_f2(ww[e]);
      }
    }
  }
  uint4 xv[C], rv[C], xn[C], rn[C];
  int row = blockIdx.x;
  if (row < M) load_row(row, xv, rv);
  for (int parity = 0; row < M; row += gridDim.x, parity ^= 1) {
    const int next = row + gridDim.x;
    if (next < M) load_row(next, xn, rn);
    if constexpr (RES) {
      __nv_bfloat16* rr = residual + static_cast<size_t>(row) * ldr;
#pragma unroll
      for (int j = 0; j < C; ++j) {
        const int c = t + T * j;
        if (c < nch) {
          uint32_t* hw = reinterpret_cast<uint32_t*>(&xv[j]);
          const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rv[j]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint64_t h = fadd2(bf16x2_to_f2(hw[e]), bf16x2_to_f2(rw[e]));
            hw[e] = pack_bf16x2(lo_f(h), hi_f(h));
          }
          *reinterpret_cast<uint4*>(rr + c * 8) = xv[j];
        }
      }
    }
    uint64_t rs2 = 0;
    if constexpr (NORM) {
      uint64_t ss2 = 0;  // (sum of even elements, sum of odd elements)
#pragma unroll
      for (int j = 0; j < C; ++j) {
        const int c = t + T * j;
        if (c < nch) {
          const uint32_t* hw = reinterpret_cast<const uint32_t*>(&xv[j]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint64_t h = bf16x2_to_f2(hw[e]);
            ss2 = fadd2(ss2, fmul2(h, h));
          }
        }
      }
      float ss = __fadd_rn(lo_f(ss2), hi_f(ss2));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      if (lane == 0) warp_ss[parity][warp] = ss;
      __syncthreads();
      ss = warp_ss[parity][0];
#pragma unroll
      for (int i = 1; i < T / 32; ++i) ss = __fadd_rn(ss, warp_ss[parity][i]);
      const float rsn = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps)));
      rs2 = pack_f2(rsn, rsn);
    }
#pragma unroll
    for (int j = 0; j < C; ++j) {
      if (T * j >= nch) break;  // uniform across the CTA
      const int c = t + T * j;
      const bool active = c < nch;
      uint32_t yw[4];  // the bf16 values to quantise, packed in pairs
      float amax = 0.f;
      if (active) {
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&xv[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (NORM) {
            const uint64_t v = fmul2(fmul2(bf16x2_to_f2(hw[e]), rs2), wf[j][e]);
            yw[e] = pack_bf16x2(lo_f(v), hi_f(v));
          } else {
            yw[e] = hw[e];
          }
        }
        const uint32_t m = bf16x2_absmax(bf16x2_absmax(yw[0], yw[1]), bf16x2_absmax(yw[2], yw[3]));
        amax = fmaxf(fabsf(__uint_as_float(m << 16)), fabsf(__uint_as_float(m & 0xffff0000u)));
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float sc = group_scale(amax);
      if (active) {
        const float nr = -__frcp_rn(sc);
        const uint64_t s2 = pack_f2(sc, sc), nr2 = pack_f2(nr, nr);
        uint32_t qw[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint64_t q0 = neg_div_by_scale2(bf16x2_to_f2(yw[2 * h]), s2, nr2);
          const uint64_t q1 = neg_div_by_scale2(bf16x2_to_f2(yw[2 * h + 1]), s2, nr2);
          qw[h] = (f2_to_e4m3x2(lo_f(q0), hi_f(q0)) | (f2_to_e4m3x2(lo_f(q1), hi_f(q1)) << 16)) ^ 0x80808080u;
        }
        *reinterpret_cast<uint2*>(A + static_cast<size_t>(row) * K + c * 8) = make_uint2(qw[0], qw[1]);
        if ((lane & 15) == 0) As[static_cast<size_t>(row) * KB + c / 16] = sc;
      }
    }
#pragma unroll
    for (int j = 0; j < C; ++j) {
      xv[j] = xn[j];
      if constexpr (RES) rv[j] = rn[j];
    }
  }
}

// The unfused chain's activation (SGLang's silu_and_mul between the gate_up GEMM and the activation quant when
// the fused kernel is off): y[m, j] = bf16(silu(g) * u) with g = gu[m, j], u = gu[m, I + j], computed in fp32
// with one rounding at the end, silu(g) = g / (1 + exp(-g)) (IEEE division, CUDA's expf). Eight columns per
// thread (16-byte loads and stores), grid-stride over the rows' 8-column chunks.
__global__ void __launch_bounds__(256) k_silu_mul(const __nv_bfloat16* __restrict__ gu, int ld_in,
                                                  __nv_bfloat16* __restrict__ y, int ld_out, int M, int I) {
  if (threadIdx.x == 0) grid_dep_launch();
  grid_dep_wait();  // gu is the previous kernel's output
  const int per_row = I / 8;
  const long long total = static_cast<long long>(M) * per_row;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / per_row);
    const int c = static_cast<int>(i - static_cast<long long>(m) * per_row) * 8;
    const __nv_bfloat16* row = gu + static_cast<size_t>(m) * ld_in;
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(row + c));
    const uint4 uv = __ldg(reinterpret_cast<const uint4*>(row + I + c));
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&uv);
    uint32_t ow[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint64_t g2 = bf16x2_to_f2(gw[e]), u2 = bf16x2_to_f2(uw[e]);
      const float g0 = lo_f(g2), g1 = hi_f(g2);
      const float y0 = __fmul_rn(__fdiv_rn(g0, __fadd_rn(1.0f, expf(-g0))), lo_f(u2));
      const float y1 = __fmul_rn(__fdiv_rn(g1, __fadd_rn(1.0f, expf(-g1))), hi_f(u2));
      ow[e] = pack_bf16x2(y0, y1);
    }
    *reinterpret_cast<uint4*>(y + static_cast<size_t>(m) * ld_out + c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// tiles[nb][kb][r][c] = W[nb*128 + r][kb*128 + c]; one CTA per 16 KB tile, 16-byte moves.
// Byte-for-byte the permute of the reference's relayout (patches/fp8_hand_sm89.py:667).
__global__ void __launch_bounds__(256) k_pack_tiles(const uint8_t* __restrict__ W, uint8_t* __restrict__ tiles, int N,
                                                   int K) {
  const int KB = K / 128;
  const long long tile = blockIdx.x;
  const long long nb = tile / KB;
  const int kb = static_cast<int>(tile - nb * KB);
  uint8_t* dst = tiles + tile * 16384;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int chunk = threadIdx.x + 256 * j;  // 1024 chunks of 16 bytes
    const int r = chunk >> 3;
    const int c16 = chunk & 7;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(W + (nb * 128 + r) * K + kb * 128 + c16 * 16));
    *reinterpret_cast<uint4*>(dst + r * 128 + c16 * 16) = v;
  }
}

}  // namespace bs

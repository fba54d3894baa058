// HBM-bound byte kernels of the path: per-token-group activation quant and the tile-first
// weight pre-pack.
#pragma once
#include "bs_common.cuh"

namespace bs {

constexpr int kQuantThreads = 256;

// x bf16 [M, K] -> A e4m3 [M, K], As fp32 [M, K/128].
// Sixteen threads own one 128-wide group (8 elements = one 16-byte load each), reduce |x| with
// shuffles inside the half-warp, then
//     As = max(amax / 448, 1e-12),  A = e4m3_rn(x / As)
// which is the reference's torch quantiser (scripts/fp8_gemm_factor_check.py:22-27:
// `s = amax / FP8_MAX; s = s.clamp_min(1e-12); (x / s).to(float8_e4m3fn)`), computed in fp32
// with IEEE division so the bytes match it exactly. |x / As| <= 448 * (1 + 2^-23), which
// rounds to 448 under both torch's conversion and the saturating cvt used here.
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
    if (active) {
      uint2 q;
      q.x = f2_to_e4m3x2(__fdiv_rn(v[0], s), __fdiv_rn(v[1], s)) |
            (f2_to_e4m3x2(__fdiv_rn(v[2], s), __fdiv_rn(v[3], s)) << 16);
      q.y = f2_to_e4m3x2(__fdiv_rn(v[4], s), __fdiv_rn(v[5], s)) |
            (f2_to_e4m3x2(__fdiv_rn(v[6], s), __fdiv_rn(v[7], s)) << 16);
      *reinterpret_cast<uint2*>(A + row * K + kb * 128 + sub * 8) = q;
      if (sub == 0) As[row * KB + kb] = s;
    }
  }
}

constexpr int kNormThreads = 256;  // one CTA per row
constexpr int kNormMaxRounds = 8;  // K <= 256 threads x 8 elements x 8 rounds = 16384

__device__ __forceinline__ void unpack_bf16x8(const uint4& raw, float (&v)[8]) {
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h2[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ float bf16_rn(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// RMSNorm followed by the per-token-group quant, one 256-thread CTA per row, without storing the bf16
// norm output. The rounding points are those of the unfused pair "RMSNorm -> per_token_group_quant_fp8":
//   h   = x                                   (or bf16_rn(x + residual), written back to residual)
//   ss  = sum of h*h in fp32 (no fused multiply-add) in a fixed order that depends on K only: thread t
//         adds the squares of its elements 8(t + 256j) + e in (j, e) order, each warp combines its lanes
//         in a butterfly (xor 16, 8, 4, 2, 1), then ss = ((w0 + w1) + w2) + ... + w7 over the 8 warps
//   rs  = 1 / sqrt(ss / K + eps)                (IEEE divide and square root)
//   y   = bf16_rn((h * rs) * w)                 (the bf16 value an unfused RMSNorm stores)
//   As  = max(amax(y over 128) / 448, 1e-12),  A = e4m3_rn(y / As)   (as k_group_quant; a 128-group is
//         the 16 chunks of one half-warp in one round)
// All of a thread's chunks (at most 8) are loaded before any is used; the second pass reads the row
// again from L1.
template <int ROUNDS>  // chunks per thread: K <= 2048 * ROUNDS
__global__ void __launch_bounds__(kNormThreads)
    k_rmsnorm_group_quant(const __nv_bfloat16* __restrict__ x, int ldx, __nv_bfloat16* residual, int ldr,
                          const __nv_bfloat16* __restrict__ w, float eps, uint8_t* __restrict__ A,
                          float* __restrict__ As, int M, int K) {
  static_assert(ROUNDS >= 1 && ROUNDS <= kNormMaxRounds, "rounds per thread");
  __shared__ float warp_ss[kNormThreads / 32];
  if (threadIdx.x == 0) grid_dep_launch();
  grid_dep_wait();  // x and the residual may be the previous kernel's output
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int row = blockIdx.x;
  const int nch = K / 8;  // 16-byte chunks in the row
  const int rounds = (nch + kNormThreads - 1) / kNormThreads;
  const __nv_bfloat16* xr = x + static_cast<size_t>(row) * ldx;
  __nv_bfloat16* rr = residual ? residual + static_cast<size_t>(row) * ldr : nullptr;

  uint4 xv[ROUNDS], rv[ROUNDS];
#pragma unroll
  for (int j = 0; j < ROUNDS; ++j) {
    const int c = j * kNormThreads + t;
    if (j < rounds && c < nch) {
      xv[j] = __ldg(reinterpret_cast<const uint4*>(xr + c * 8));
      if (rr) rv[j] = *reinterpret_cast<const uint4*>(rr + c * 8);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < ROUNDS; ++j) {
    const int c = j * kNormThreads + t;
    if (j < rounds && c < nch) {
      float h[8];
      unpack_bf16x8(xv[j], h);
      if (rr) {
        float r8[8];
        unpack_bf16x8(rv[j], r8);
        uint32_t packed[4];
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = bf16_rn(__fadd_rn(h[e], r8[e]));
#pragma unroll
        for (int e = 0; e < 4; ++e) packed[e] = pack_bf16x2(h[2 * e], h[2 * e + 1]);
        xv[j] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        *reinterpret_cast<uint4*>(rr + c * 8) = xv[j];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(h[e], h[e]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  if (lane == 0) warp_ss[t >> 5] = ss;
  __syncthreads();
  ss = warp_ss[0];
#pragma unroll
  for (int i = 1; i < kNormThreads / 32; ++i) ss = __fadd_rn(ss, warp_ss[i]);
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps)));

  const int KB = K / 128;
#pragma unroll
  for (int j = 0; j < ROUNDS; ++j) {
    if (j >= rounds) break;  // uniform across the CTA
    const int c = j * kNormThreads + t;
    const bool active = c < nch;
    float y[8];
    if (active) {
      float h[8], wf[8];
      unpack_bf16x8(xv[j], h);  // h (the residual sum when fused) is still in registers
      unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(w + c * 8)), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = bf16_rn(__fmul_rn(__fmul_rn(h[e], rs), wf[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(y[e]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = fmaxf(__fdiv_rn(amax, 448.0f), 1e-12f);
    if (active) {
      uint2 q;
      q.x = f2_to_e4m3x2(__fdiv_rn(y[0], sc), __fdiv_rn(y[1], sc)) |
            (f2_to_e4m3x2(__fdiv_rn(y[2], sc), __fdiv_rn(y[3], sc)) << 16);
      q.y = f2_to_e4m3x2(__fdiv_rn(y[4], sc), __fdiv_rn(y[5], sc)) |
            (f2_to_e4m3x2(__fdiv_rn(y[6], sc), __fdiv_rn(y[7], sc)) << 16);
      *reinterpret_cast<uint2*>(A + static_cast<size_t>(row) * K + c * 8) = q;
      if ((lane & 15) == 0) As[static_cast<size_t>(row) * KB + c / 16] = sc;
    }
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

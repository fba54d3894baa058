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

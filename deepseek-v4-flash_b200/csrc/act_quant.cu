// act_quant.cu -- 1 x block FP8 e4m3 activation quantisation.
//
// Replaces kernel.act_quant (Deepseek_origin/inference/kernel.py:105-125,
// TileLang kernel :40-102).  Semantics, bit-exact with the reference:
//   amax = max(max |x| over the block, 1e-4)                 (kernel.py:77-79)
//   s    = amax / 448, correctly rounded                   (kernel_fallback.py:27-28)
//        or, with round_scale, 2^(exponent(s) + (mantissa(s) != 0))
//                                                          (kernel.py:22-37)
//   y    = e4m3_rne(clamp(x / s, -448, 448))               (kernel.py:93-96)
//   inplace: x = bf16(f32(y) * s)                          (kernel.py:84-91)
//
// HBM-bound byte work: one warp per (row, block); each lane owns block/32
// consecutive bf16 values, so a warp reads the block as one coalesced run and
// writes its codes as one coalesced run.
#include "common.cuh"
#include "kernels.h"

namespace qcau {

template <int kPer>  // values per lane = block / 32
__global__ void act_quant_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ y,
                                 void* __restrict__ s, __nv_bfloat16* __restrict__ x_inplace,
                                 int64_t m, int64_t n, int round_scale, int scale_e8m0) {
  constexpr int kBlock = kPer * 32;
  const int lane = threadIdx.x & 31;
  const int64_t nb = n / kBlock;
  const int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (task >= m * nb) return;
  const int64_t row = task / nb, blk = task % nb;
  const int64_t base = row * n + blk * kBlock + lane * kPer;

  float v[kPer];
  const __nv_bfloat16* src = x_inplace ? x_inplace : x;
  if constexpr (kPer == 4) {
    uint2 raw = *reinterpret_cast<const uint2*>(src + base);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = __bfloat162float(h[i]);
  } else if constexpr (kPer == 2) {
    uint32_t raw = *reinterpret_cast<const uint32_t*>(src + base);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
    v[0] = __bfloat162float(h[0]);
    v[1] = __bfloat162float(h[1]);
  } else {
#pragma unroll
    for (int i = 0; i < kPer; i++) v[i] = __bfloat162float(src[base + i]);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; i++) amax = fmaxf(amax, fabsf(v[i]));
  amax = warp_max(amax);
  const float sc = act_scale(amax, round_scale);

  uint8_t code[kPer];
#pragma unroll
  for (int i = 0; i < kPer; i++) {
    float q = __fdiv_rn(v[i], sc);
    q = fminf(fmaxf(q, -448.f), 448.f);
    code[i] = f32_to_e4m3(q);
  }
  if (x_inplace) {
#pragma unroll
    for (int i = 0; i < kPer; i++)
      x_inplace[base + i] = __float2bfloat16_rn(__fmul_rn(e4m3_to_f32(code[i]), sc));
    return;
  }
  if constexpr (kPer == 4) {
    uint32_t packed = (uint32_t)code[0] | ((uint32_t)code[1] << 8) | ((uint32_t)code[2] << 16) |
                      ((uint32_t)code[3] << 24);
    *reinterpret_cast<uint32_t*>(y + base) = packed;
  } else {
#pragma unroll
    for (int i = 0; i < kPer; i++) y[base + i] = code[i];
  }
  if (lane == 0) {
    const int64_t si = row * nb + blk;
    if (scale_e8m0)
      reinterpret_cast<uint8_t*>(s)[si] = (uint8_t)((__float_as_uint(sc) >> 23) & 0xff);
    else
      reinterpret_cast<float*>(s)[si] = sc;
  }
}

cudaError_t launch_act_quant(const void* x, void* y, void* s, int64_t m, int64_t n, int block,
                             int round_scale, int scale_e8m0, int inplace, cudaStream_t st) {
  const int64_t tasks = m * (n / block);
  if (tasks == 0) return cudaSuccess;
  const int warps = 8;
  const unsigned grid = (unsigned)((tasks + warps - 1) / warps);
  auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* xi = inplace ? reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(x)) : nullptr;
  auto* yb = reinterpret_cast<uint8_t*>(y);
  switch (block) {
    case 128:
      act_quant_kernel<4><<<grid, warps * 32, 0, st>>>(xb, yb, s, xi, m, n, round_scale,
                                                       scale_e8m0);
      break;
    case 64:
      act_quant_kernel<2><<<grid, warps * 32, 0, st>>>(xb, yb, s, xi, m, n, round_scale,
                                                       scale_e8m0);
      break;
    case 32:
      act_quant_kernel<1><<<grid, warps * 32, 0, st>>>(xb, yb, s, xi, m, n, round_scale,
                                                       scale_e8m0);
      break;
    case 256:
      act_quant_kernel<8><<<grid, warps * 32, 0, st>>>(xb, yb, s, xi, m, n, round_scale,
                                                       scale_e8m0);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// FP8 weight with 128 x 128 block scales -> bf16 (one-time weight preparation
// of wkv_b for the absorbed decode layer).
__global__ void dequant_fp8_weight_kernel(const uint8_t* __restrict__ w, const void* __restrict__ s,
                                          int scale_e8m0, __nv_bfloat16* __restrict__ out,
                                          int64_t rows, int64_t cols) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i % cols;
  const int64_t sc_cols = (cols + 127) / 128;
  const float sc = load_scale(s, (r / 128) * sc_cols + c / 128, scale_e8m0);
  out[i] = __float2bfloat16_rn(__fmul_rn(e4m3_to_f32(w[i]), sc));
}

cudaError_t launch_dequant_fp8_weight(const void* w, const void* s, int scale_e8m0, void* out,
                                      int64_t rows, int64_t cols, cudaStream_t st) {
  const int64_t n = rows * cols;
  if (n == 0) return cudaSuccess;
  dequant_fp8_weight_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const uint8_t*>(w), s, scale_e8m0,
      reinterpret_cast<__nv_bfloat16*>(out), rows, cols);
  return cudaGetLastError();
}

}  // namespace qcau

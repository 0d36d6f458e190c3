// gemm_epilogue.cuh - the fused GEMM epilogue shared by the 1-SM and 2-SM
// tcgen05 GEMM kernels: bias, tanh-GELU, RoPE and residual in registers,
// per-thread stores or swizzled staging for TMA stores.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemm_sm100.cuh"

namespace s3 {
namespace {

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5*x*(1+tanh(sqrt(2/pi)*(x+0.044715x^3))), cpu_gelu.c:23-36
  float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}

// Same formula with the SFU's tanh.approx.f32 (max relative error about
// 2^-11, below the 2^-9 rounding of the 16-bit outputs it is used for).
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(inner));
  return 0.5f * x * (1.0f + t);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Bias, activation and RoPE on 32 consecutive columns [col0, col0+32) of
// one output row, in registers.
__device__ __forceinline__ void epilogue_math(const EpiParams& ep, float (&v)[32], int row, int col0,
                                              int N, bool add_bias = true) {
  const bool full = col0 + 32 <= N;
  if (ep.col_scale) {
    if (full) {
      const float4* s4 = reinterpret_cast<const float4*>(ep.col_scale + col0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 c = __ldg(s4 + j);
        v[4 * j] *= c.x;
        v[4 * j + 1] *= c.y;
        v[4 * j + 2] *= c.z;
        v[4 * j + 3] *= c.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] *= __ldg(ep.col_scale + col0 + j);
    }
  }
  if (ep.bias && add_bias) {
    if (full) {
      const float4* b4 = reinterpret_cast<const float4*>(ep.bias + col0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 b = __ldg(b4 + j);
        v[4 * j] += b.x;
        v[4 * j + 1] += b.y;
        v[4 * j + 2] += b.z;
        v[4 * j + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] += __ldg(ep.bias + col0 + j);
    }
  }
  if (ep.act == 1) {
    if (ep.out_type == kOutF32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh_fast(v[j]);
    }
  }
  if (col0 < ep.rope_cols) {
    const int p = row % ep.rope_period;
    const float2* cs = ep.rope_cs + static_cast<int64_t>((col0 & 63) >> 1) * ep.rope_period + p;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 t = __ldg(cs + static_cast<int64_t>(i) * ep.rope_period);
      const float x0 = v[2 * i], x1 = v[2 * i + 1];
      v[2 * i] = x0 * t.x - x1 * t.y;
      v[2 * i + 1] = x0 * t.y + x1 * t.x;
    }
  }
}

// v += residual row (row % res_row_period when periodic), in registers.
__device__ __forceinline__ void epilogue_residual(const EpiParams& ep, float (&v)[32], int row, int col0, int N) {
  const bool full = col0 + 32 <= N;
  {
    int rr = ep.res_row_period > 0 ? row % ep.res_row_period : row;
    const float* r = ep.residual + static_cast<int64_t>(rr) * ep.ldr + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 x = *reinterpret_cast<const float4*>(r + 4 * j);
        v[4 * j] += x.x;
        v[4 * j + 1] += x.y;
        v[4 * j + 2] += x.z;
        v[4 * j + 3] += x.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] += r[j];
    }
  }
}

// Residual add and per-thread store of the same 32 columns (kEpiDirect).
__device__ __forceinline__ void epilogue_store_direct(const EpiParams& ep, float (&v)[32], int row,
                                                      int col0, int N) {
  const bool full = col0 + 32 <= N;
  if (ep.residual) epilogue_residual(ep, v, row, col0, N);
  int orow = row;
  if (ep.out_row_map) {
    int per = ep.out_row_period;
    orow = (row / per) * per + __ldg(ep.out_row_map + row % per);
  }
  const int64_t off = static_cast<int64_t>(orow) * ep.ldo + col0;
  if (ep.out_type == kOutF32) {
    float* o = static_cast<float*>(ep.out) + off;
    if (full) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        reinterpret_cast<float4*>(o)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) o[j] = v[j];
    }
  } else {
    const bool bf = ep.out_type == kOutBF16;
    uint16_t* o = static_cast<uint16_t*>(ep.out) + off;
    if (full) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 w;
        w.x = bf ? pack_bf16(v[8 * j], v[8 * j + 1]) : pack_f16(v[8 * j], v[8 * j + 1]);
        w.y = bf ? pack_bf16(v[8 * j + 2], v[8 * j + 3]) : pack_f16(v[8 * j + 2], v[8 * j + 3]);
        w.z = bf ? pack_bf16(v[8 * j + 4], v[8 * j + 5]) : pack_f16(v[8 * j + 4], v[8 * j + 5]);
        w.w = bf ? pack_bf16(v[8 * j + 6], v[8 * j + 7]) : pack_f16(v[8 * j + 6], v[8 * j + 7]);
        reinterpret_cast<uint4*>(o)[j] = w;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) {
          uint16_t h;
          if (bf) {
            __nv_bfloat16 t = __float2bfloat16_rn(v[j]);
            h = *reinterpret_cast<uint16_t*>(&t);
          } else {
            __half t = __float2half_rn(v[j]);
            h = *reinterpret_cast<uint16_t*>(&t);
          }
          o[j] = h;
        }
    }
  }
}

// Write one thread's 32 values (row `lane` of a 32x32 chunk) into the
// warp's staging buffer in the layout of the output tensor map: f32 rows of
// 128 B with the 128-byte swizzle, or 16-bit rows of 64 B with the 64-byte
// swizzle (16-byte chunk c of row r lands at c ^ (r & 7), resp.
// c ^ ((r >> 1) & 3)), which keeps the 16-byte stores bank-conflict free.
__device__ __forceinline__ void stage_chunk(uint8_t* buf, const float (&v)[32], int lane, int out_type) {
  if (out_type == kOutF32) {
    uint8_t* rowp = buf + lane * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(rowp + ((c ^ (lane & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  } else {
    const bool bf = out_type == kOutBF16;
    uint8_t* rowp = buf + lane * 64;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 w;
      w.x = bf ? pack_bf16(v[8 * c], v[8 * c + 1]) : pack_f16(v[8 * c], v[8 * c + 1]);
      w.y = bf ? pack_bf16(v[8 * c + 2], v[8 * c + 3]) : pack_f16(v[8 * c + 2], v[8 * c + 3]);
      w.z = bf ? pack_bf16(v[8 * c + 4], v[8 * c + 5]) : pack_f16(v[8 * c + 4], v[8 * c + 5]);
      w.w = bf ? pack_bf16(v[8 * c + 6], v[8 * c + 7]) : pack_f16(v[8 * c + 6], v[8 * c + 7]);
      *reinterpret_cast<uint4*>(rowp + ((c ^ ((lane >> 1) & 3)) << 4)) = w;
    }
  }
}

}  // namespace
}  // namespace s3

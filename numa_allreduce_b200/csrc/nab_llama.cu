// Decode-step kernels of the tensor-parallel Llama model (no counterpart in
// the reference, which has no model code):
//   rope_append   rotary embedding of this rank's q and k heads (half-split
//                 convention) and append of k, v at the current position of
//                 the KV cache; the position is read from device memory so a
//                 captured CUDA graph replays at any position;
//   attention     GQA decode attention, split over the sequence: one CTA per
//                 (batch, kv head, split) with one warp per query head of the
//                 group; K/V of a chunk staged in shared memory; partial
//                 (max, sum, output) combined by a second kernel;
//   silu_mul      SwiGLU gating of the fused gate|up projection.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "nab_device.cuh"
#include "nab_llama.h"

namespace nab {

namespace {

constexpr int kHeadDim = 128;
constexpr int kChunk = 64;  // positions per attention split

NAB_DINLINE float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }

// grid (B, Hq + 2 * Hkv), block kHeadDim / 2 threads.
__global__ void k_rope_append(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t,
                              const float* __restrict__ sin_t, const int* __restrict__ pos_ptr,
                              __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                              __nv_bfloat16* __restrict__ v_cache, int Hq, int Hkv, int Lmax) {
  const int b = blockIdx.x, h = blockIdx.y, i = threadIdx.x;  // i < 64
  const int pos = *pos_ptr;
  const int width = (Hq + 2 * Hkv) * kHeadDim;
  const __nv_bfloat16* src = qkv + static_cast<int64_t>(b) * width + h * kHeadDim;
  const float x1 = bf2f(src[i]), x2 = bf2f(src[i + kHeadDim / 2]);
  if (h < Hq + Hkv) {
    const float c = cos_t[pos * (kHeadDim / 2) + i], s = sin_t[pos * (kHeadDim / 2) + i];
    const float y1 = x1 * c - x2 * s, y2 = x2 * c + x1 * s;
    __nv_bfloat16* dst;
    if (h < Hq) {
      dst = q_out + (static_cast<int64_t>(b) * Hq + h) * kHeadDim;
    } else {
      dst = k_cache + ((static_cast<int64_t>(b) * Hkv + (h - Hq)) * Lmax + pos) * kHeadDim;
    }
    dst[i] = __float2bfloat16_rn(y1);
    dst[i + kHeadDim / 2] = __float2bfloat16_rn(y2);
  } else {
    __nv_bfloat16* dst = v_cache + ((static_cast<int64_t>(b) * Hkv + (h - Hq - Hkv)) * Lmax + pos) * kHeadDim;
    dst[i] = src[i];
    dst[i + kHeadDim / 2] = src[i + kHeadDim / 2];
  }
}

// grid (B, Hkv, splits), block 32 * G threads (G = Hq / Hkv query heads per kv head).
// Writes per (b, q head, split): m (running max), l (sum of exp) and the
// unnormalised output accumulator.
__global__ void __launch_bounds__(256) k_attn_partial(const __nv_bfloat16* __restrict__ q,
                                                      const __nv_bfloat16* __restrict__ k_cache,
                                                      const __nv_bfloat16* __restrict__ v_cache,
                                                      const int* __restrict__ pos_ptr, float* __restrict__ part_ml,
                                                      float* __restrict__ part_o, int Hq, int Hkv, int Lmax,
                                                      int splits, float scale) {
  __shared__ __align__(16) __nv_bfloat16 sk[kChunk][kHeadDim + 8];
  __shared__ __align__(16) __nv_bfloat16 sv[kChunk][kHeadDim + 8];
  const int b = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = kvh * G + warp;
  const int L = *pos_ptr + 1;
  const int per = (L + splits - 1) / splits;
  const int beg = sp * per, end = min(L, beg + per);
  // q of this warp's head: lane holds dims lane*4 .. lane*4+3
  float qv[4];
  {
    const __nv_bfloat16* qp = q + (static_cast<int64_t>(b) * Hq + h) * kHeadDim + lane * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) qv[e] = bf2f(qp[e]) * scale;
  }
  float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  const __nv_bfloat16* kb = k_cache + (static_cast<int64_t>(b) * Hkv + kvh) * Lmax * kHeadDim;
  const __nv_bfloat16* vb = v_cache + (static_cast<int64_t>(b) * Hkv + kvh) * Lmax * kHeadDim;
  for (int c0 = beg; c0 < end; c0 += kChunk) {
    const int n = min(kChunk, end - c0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < n * (kHeadDim / 8); idx += blockDim.x) {
      const int r = idx / (kHeadDim / 8), cc = (idx % (kHeadDim / 8)) * 8;
      *reinterpret_cast<uint4*>(&sk[r][cc]) = *reinterpret_cast<const uint4*>(kb + static_cast<int64_t>(c0 + r) * kHeadDim + cc);
      *reinterpret_cast<uint4*>(&sv[r][cc]) = *reinterpret_cast<const uint4*>(vb + static_cast<int64_t>(c0 + r) * kHeadDim + cc);
    }
    __syncthreads();
    if (warp < G) {
      for (int j = 0; j < n; ++j) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) d += qv[e] * bf2f(sk[j][lane * 4 + e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        const float mn = fmaxf(m, d);
        const float corr = __expf(m - mn);
        const float p = __expf(d - mn);
        l = l * corr + p;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = acc[e] * corr + p * bf2f(sv[j][lane * 4 + e]);
        m = mn;
      }
    }
  }
  if (warp < G) {
    const int64_t idx = (static_cast<int64_t>(b) * Hq + h) * splits + sp;
    if (lane == 0) {
      part_ml[idx * 2] = m;
      part_ml[idx * 2 + 1] = l;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) part_o[idx * kHeadDim + lane * 4 + e] = acc[e];
  }
}

// grid (B, Hq), block kHeadDim threads.
__global__ void k_attn_combine(const float* __restrict__ part_ml, const float* __restrict__ part_o,
                               __nv_bfloat16* __restrict__ out, int Hq, int splits) {
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int64_t base = (static_cast<int64_t>(b) * Hq + h) * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(base + s) * 2]);
  float den = 0.f, num = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = part_ml[(base + s) * 2];
    if (ms == -INFINITY) continue;
    const float w = __expf(ms - M);
    den += w * part_ml[(base + s) * 2 + 1];
    num += w * part_o[(base + s) * kHeadDim + d];
  }
  out[(static_cast<int64_t>(b) * Hq + h) * kHeadDim + d] = __float2bfloat16_rn(num / den);
}

// out[b, i] = silu(gu[b, i]) * gu[b, I + i]
__global__ void k_silu_mul(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int B, int I) {
  const int64_t n = static_cast<int64_t>(B) * I;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = t / I, i = t % I;
    const float g = bf2f(gu[b * 2 * I + i]), u = bf2f(gu[b * 2 * I + I + i]);
    out[t] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * u);
  }
}

void check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

void rope_append(cudaStream_t s, const void* qkv, const float* cos_t, const float* sin_t, const int* pos,
                 void* q_out, void* k_cache, void* v_cache, int B, int Hq, int Hkv, int Lmax) {
  k_rope_append<<<dim3(B, Hq + 2 * Hkv), kHeadDim / 2, 0, s>>>(
      static_cast<const __nv_bfloat16*>(qkv), cos_t, sin_t, pos, static_cast<__nv_bfloat16*>(q_out),
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), Hq, Hkv, Lmax);
  check("rope_append");
}

void decode_attention(cudaStream_t s, const void* q, const void* k_cache, const void* v_cache, const int* pos,
                      float* part_ml, float* part_o, void* out, int B, int Hq, int Hkv, int Lmax, int splits) {
  if (Hq % Hkv != 0 || Hq / Hkv > 8) throw std::invalid_argument("attention: need Hq / Hkv <= 8");
  const float scale = 1.f / sqrtf(static_cast<float>(kHeadDim));
  k_attn_partial<<<dim3(B, Hkv, splits), 32 * (Hq / Hkv), 0, s>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k_cache),
      static_cast<const __nv_bfloat16*>(v_cache), pos, part_ml, part_o, Hq, Hkv, Lmax, splits, scale);
  check("attention partial");
  k_attn_combine<<<dim3(B, Hq), kHeadDim, 0, s>>>(part_ml, part_o, static_cast<__nv_bfloat16*>(out), Hq, splits);
  check("attention combine");
}

void silu_mul(cudaStream_t s, const void* gu, void* out, int B, int I) {
  const int64_t n = static_cast<int64_t>(B) * I;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
  k_silu_mul<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), B, I);
  check("silu_mul");
}

}  // namespace nab

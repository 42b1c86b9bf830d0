// Decode-step kernels of the tensor-parallel Llama model (no counterpart in
// the reference, which has no model code):
//   rope_append   rotary embedding of this rank's q and k heads (half-split
//                 convention) and append of k, v at the current position of
//                 the KV cache; the position is read from device memory so a
//                 captured CUDA graph replays at any position;
//   attention     GQA decode attention, split over the sequence: one CTA per
//                 (batch, kv head, split) with one warp per query head of the
//                 group; K/V of a chunk staged in shared memory; the last CTA
//                 of each (batch, kv head) combines the partial (max, sum,
//                 output) of all splits in the same launch;
//   silu_mul      SwiGLU gating of the fused gate|up projection.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
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
  pdl_trigger();
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

// grid (B, Hkv, splits), block 32 * G threads (G = Hq / Hkv query heads per
// kv head, one warp each). Each CTA covers one contiguous range of positions:
// K/V rows are staged in shared memory 64 at a time, every warp scores four
// positions per step (four independent shuffle reductions in flight) and
// keeps an online softmax (running max m, sum l, unnormalised output).
// The partial (m, l, o) of every (b, head, split) goes to scratch; the last
// CTA of a (b, kv head) to finish (arrival counter, reset by that CTA) combines
// the splits of its G heads and writes the output, so one launch does both.
__global__ void __launch_bounds__(256) k_attn_decode(const __nv_bfloat16* __restrict__ q,
                                                     const __nv_bfloat16* __restrict__ k_cache,
                                                     const __nv_bfloat16* __restrict__ v_cache,
                                                     const int* __restrict__ pos_ptr, float* __restrict__ part_ml,
                                                     float* __restrict__ part_o, int* __restrict__ counters,
                                                     __nv_bfloat16* __restrict__ out, int Hq, int Hkv, int Lmax,
                                                     int splits, float scale) {
  pdl_trigger();
  __shared__ __align__(16) __nv_bfloat16 sk[kChunk][kHeadDim + 8];
  __shared__ __align__(16) __nv_bfloat16 sv[kChunk][kHeadDim + 8];
  __shared__ int s_last;
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
    const uint2 raw = *reinterpret_cast<const uint2*>(q + (static_cast<int64_t>(b) * Hq + h) * kHeadDim + lane * 4);
    const __nv_bfloat162 q01 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 q23 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    qv[0] = __low2float(q01) * scale;
    qv[1] = __high2float(q01) * scale;
    qv[2] = __low2float(q23) * scale;
    qv[3] = __high2float(q23) * scale;
  }
  float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  const __nv_bfloat16* kb = k_cache + (static_cast<int64_t>(b) * Hkv + kvh) * Lmax * kHeadDim;
  const __nv_bfloat16* vb = v_cache + (static_cast<int64_t>(b) * Hkv + kvh) * Lmax * kHeadDim;
  auto row4 = [&](const __nv_bfloat16* r, float (&f)[4]) {
    const uint2 raw = *reinterpret_cast<const uint2*>(r + lane * 4);
    const __nv_bfloat162 a0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 a1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    f[0] = __low2float(a0);
    f[1] = __high2float(a0);
    f[2] = __low2float(a1);
    f[3] = __high2float(a1);
  };
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
      for (int j = 0; j < n; j += 4) {
        float d[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float kf[4];
          row4(sk[min(j + u, n - 1)], kf);
          d[u] = qv[0] * kf[0] + qv[1] * kf[1] + qv[2] * kf[2] + qv[3] * kf[3];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int u = 0; u < 4; ++u) d[u] += __shfl_xor_sync(0xffffffffu, d[u], o);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j + u >= n) d[u] = -INFINITY;
        const float mn = fmaxf(fmaxf(m, fmaxf(d[0], d[1])), fmaxf(d[2], d[3]));
        const float corr = __expf(m - mn);
        float p[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) p[u] = __expf(d[u] - mn);
        l = l * corr + ((p[0] + p[1]) + (p[2] + p[3]));
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] *= corr;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float vf[4];
          row4(sv[min(j + u, n - 1)], vf);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[e] += p[u] * vf[e];
        }
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
    *reinterpret_cast<float4*>(part_o + idx * kHeadDim + lane * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
  // last split CTA of this (b, kv head) combines
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ctr = counters + b * Hkv + kvh;
    s_last = atomicAdd(ctr, 1) == splits - 1;
    if (s_last) *ctr = 0;
  }
  __syncthreads();
  if (!s_last || warp >= G) return;
  __threadfence();
  const int64_t base = (static_cast<int64_t>(b) * Hq + h) * splits;
  float M = -INFINITY;
  for (int s2 = 0; s2 < splits; ++s2) M = fmaxf(M, __ldcg(part_ml + (base + s2) * 2));
  float den = 0.f, num[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s2 = 0; s2 < splits; ++s2) {
    const float ms = __ldcg(part_ml + (base + s2) * 2);
    if (ms == -INFINITY) continue;
    const float w = __expf(ms - M);
    den += w * __ldcg(part_ml + (base + s2) * 2 + 1);
    const float4 o = __ldcg(reinterpret_cast<const float4*>(part_o + (base + s2) * kHeadDim + lane * 4));
    num[0] += w * o.x;
    num[1] += w * o.y;
    num[2] += w * o.z;
    num[3] += w * o.w;
  }
  const float inv = 1.f / den;
  __nv_bfloat162 o01 = __floats2bfloat162_rn(num[0] * inv, num[1] * inv);
  __nv_bfloat162 o23 = __floats2bfloat162_rn(num[2] * inv, num[3] * inv);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&o01);
  packed.y = *reinterpret_cast<uint32_t*>(&o23);
  *reinterpret_cast<uint2*>(out + (static_cast<int64_t>(b) * Hq + h) * kHeadDim + lane * 4) = packed;
}

// out[b, i] = silu(gu[b, i]) * gu[b, I + i]
__global__ void k_silu_mul(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int B, int I) {
  pdl_trigger();
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
                      float* part_ml, float* part_o, int* counters, void* out, int B, int Hq, int Hkv, int Lmax,
                      int splits) {
  if (Hq % Hkv != 0 || Hq / Hkv > 8) throw std::invalid_argument("attention: need Hq / Hkv <= 8");
  const float scale = 1.f / sqrtf(static_cast<float>(kHeadDim));
  k_attn_decode<<<dim3(B, Hkv, splits), 32 * (Hq / Hkv), 0, s>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k_cache),
      static_cast<const __nv_bfloat16*>(v_cache), pos, part_ml, part_o, counters,
      static_cast<__nv_bfloat16*>(out), Hq, Hkv, Lmax, splits, scale);
  check("attention");
}

int attention_splits(int B, int Hkv, int context, int sms) {
  // about two CTAs per SM, at least 16 positions per split
  const int want = std::max(1, (2 * sms) / std::max(1, B * Hkv));
  const int most = std::max(1, (context + 15) / 16);
  return std::max(1, std::min({want, most, 128}));
}

void silu_mul(cudaStream_t s, const void* gu, void* out, int B, int I) {
  const int64_t n = static_cast<int64_t>(B) * I;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
  k_silu_mul<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), B, I);
  check("silu_mul");
}

}  // namespace nab

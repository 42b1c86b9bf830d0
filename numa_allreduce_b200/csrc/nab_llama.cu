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
#include "nab_driver.h"
#include "nab_kerr.h"
#include "nab_llama.h"
#include "nab_sm100.cuh"

namespace nab {

namespace {

constexpr int kHeadDim = 128;
constexpr int kChunk = 64;           // K/V rows staged per step
constexpr int kMaxAttnSplits = 16;  // CTAs per (batch, kv head): one cluster
constexpr int kAttnSmem = 2 * 2 * kChunk * kHeadDim * 2;  // 2 stages of K and V chunks

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

struct AttnArgs {
  const __nv_bfloat16* q;  // [B, q_stride]: q heads at 0 (kRope: the qkv projection)
  const float* cos_t;      // kRope: [Lmax, 64]
  const float* sin_t;
  const int* pos;          // position being decoded (device memory)
  __nv_bfloat16* k_cache;  // [B, Hkv, Lmax, 128]
  __nv_bfloat16* v_cache;
  __nv_bfloat16* out;      // [B, Hq, 128]
  int q_stride;
  int Hq, Hkv, Lmax, splits;
  float scale;
  ErrorState* err;         // the device's kernel error record
  uint32_t* err_host;
  uint64_t timeout_ns;
};

NAB_DINLINE uint2 pack4(const float (&f)[4]) {
  __nv_bfloat162 a0 = __floats2bfloat162_rn(f[0], f[1]), a1 = __floats2bfloat162_rn(f[2], f[3]);
  uint2 r;
  r.x = *reinterpret_cast<uint32_t*>(&a0);
  r.y = *reinterpret_cast<uint32_t*>(&a1);
  return r;
}

// GQA decode attention. grid (splits, B * Hkv); the `splits` CTAs of one
// (batch, kv head) form a thread-block cluster and each covers one
// contiguous range of positions. Block: one warp per query head of the group
// (G = Hq / Hkv <= 8); lane l holds dims 4l..4l+3. K/V rows of the range are
// contiguous in the cache, so each 64-row chunk arrives by two bulk copies
// (TMA) into a 2-stage shared-memory ring while the previous chunk is
// scored; every warp scores four positions per step (four independent
// shuffle reductions in flight) with an online softmax (running max m, sum
// l, unnormalised output). Each CTA leaves its partial in shared memory;
// after a cluster barrier CTA 0 combines the splits over distributed shared
// memory and writes the output: one launch, no scratch.
// kRope: q and the new k are rotated here from the qkv projection; the CTA
// holding the current position writes k and v to the cache and into its
// staged chunk.
template <bool kRope>
__global__ void __launch_bounds__(256) k_attn(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  // [stage][K | V][kChunk][kHeadDim] bf16
  auto kv_tile = [&](int stage, int which) {
    return reinterpret_cast<__nv_bfloat16*>(attn_smem) + (stage * 2 + which) * kChunk * kHeadDim;
  };
  __shared__ __align__(16) float s_o[8][kHeadDim];
  __shared__ float s_m[8], s_l[8];
  __shared__ __align__(8) uint64_t full_bar[2];
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int sp = blockIdx.x, b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = kvh * G + warp;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&full_bar[0], 1);
    sm100::mbar_init(&full_bar[1], 1);
    sm100::fence_barrier_init();
    s_abort = 0;
  }
  __syncthreads();
  sm100::griddep_wait();  // inputs come from the kernel before (programmatic launch)
  pdl_trigger();
  const int pos = *a.pos;
  const int L = pos + 1;
  const int per = (L + a.splits - 1) / a.splits;
  const int beg = sp * per, end = min(L, beg + per);
  const int nchunks = end > beg ? (end - beg + kChunk - 1) / kChunk : 0;
  const int64_t kv_base = (static_cast<int64_t>(b) * a.Hkv + kvh) * a.Lmax * kHeadDim;
  const __nv_bfloat16* kb = a.k_cache + kv_base;
  const __nv_bfloat16* vb = a.v_cache + kv_base;
  int issued = 0;  // chunks whose copies thread 0 started
  auto issue = [&](int i) {  // chunk i into stage i & 1 (thread 0)
    ++issued;
    const int c0 = beg + i * kChunk, n = min(kChunk, end - c0);
    const uint32_t bytes = static_cast<uint32_t>(n) * kHeadDim * 2;
    sm100::mbar_arrive_expect_tx(&full_bar[i & 1], 2 * bytes);
    sm100::bulk_load(kv_tile(i & 1, 0), kb + static_cast<int64_t>(c0) * kHeadDim, bytes, &full_bar[i & 1]);
    sm100::bulk_load(kv_tile(i & 1, 1), vb + static_cast<int64_t>(c0) * kHeadDim, bytes, &full_bar[i & 1]);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(2, nchunks); ++i) issue(i);

  // Lane = (group g = lane / 8, slice s = lane % 8). Group g scores the
  // positions j + g of each step of 4; slice s holds dims 8s..8s+7 and
  // 64+8s..64+8s+7 (a rotary pair sits in one lane; the 8 lanes of a group
  // read one contiguous 256-byte K/V row without bank conflicts).
  const int g = lane >> 3, sl = lane & 7;
  const int d0 = 8 * sl, d1 = 64 + 8 * sl;
  const __nv_bfloat16* qrow = a.q + static_cast<int64_t>(b) * a.q_stride;
  auto load8 = [](const __nv_bfloat16* p, float* f) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      f[2 * k] = __uint_as_float(w[k] << 16);
      f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  };
  auto store8 = [](__nv_bfloat16* p, const float* f) {
    uint4 r;
    uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t*>(&t);
    }
    *reinterpret_cast<uint4*>(p) = r;
  };
  // half-split rotary embedding of dims (d0 + e, d1 + e), both in this lane
  auto rope16 = [&](float* x) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float c = a.cos_t[pos * (kHeadDim / 2) + d0 + e], sn = a.sin_t[pos * (kHeadDim / 2) + d0 + e];
      const float x1 = x[e], x2 = x[8 + e];
      x[e] = x1 * c - x2 * sn;
      x[8 + e] = x2 * c + x1 * sn;
    }
  };
  float qv[16];
  if (warp < G) {
    load8(qrow + h * kHeadDim + d0, qv);
    load8(qrow + h * kHeadDim + d1, qv + 8);
    if (kRope) {
      rope16(qv);
#pragma unroll
      for (int e = 0; e < 16; ++e) qv[e] = __bfloat162float(__float2bfloat16_rn(qv[e]));  // as rope_append stores q
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) qv[e] *= a.scale;
  }
  // the new position's k (rotated) and v: to the cache, and into the staged
  // chunk below (the bulk copy may have read the row before this store);
  // lanes 0-7 of warp 0 hold them
  const bool owns_pos = kRope && beg <= pos && pos < end;
  float k_new[16], v_new[16];
  if (owns_pos && warp == 0 && g == 0) {
    load8(qrow + (a.Hq + kvh) * kHeadDim + d0, k_new);
    load8(qrow + (a.Hq + kvh) * kHeadDim + d1, k_new + 8);
    rope16(k_new);
    load8(qrow + (a.Hq + a.Hkv + kvh) * kHeadDim + d0, v_new);
    load8(qrow + (a.Hq + a.Hkv + kvh) * kHeadDim + d1, v_new + 8);
    const int64_t at = kv_base + static_cast<int64_t>(pos) * kHeadDim;
    store8(a.k_cache + at + d0, k_new);
    store8(a.k_cache + at + d1, k_new + 8);
    store8(a.v_cache + at + d0, v_new);
    store8(a.v_cache + at + d1, v_new + 8);
  }

  float m = -INFINITY, l = 0.f, acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
  // one position of this group: score, then the online-softmax update
  auto score = [&](const __nv_bfloat16* krow) {
    float kf[16];
    load8(krow + d0, kf);
    load8(krow + d1, kf + 8);
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      s0 += qv[e] * kf[e];
      s1 += qv[e + 1] * kf[e + 1];
      s2 += qv[e + 2] * kf[e + 2];
      s3 += qv[e + 3] * kf[e + 3];
    }
    return (s0 + s1) + (s2 + s3);
  };
  auto update = [&](float d, const __nv_bfloat16* vrow) {
    float vf[16];
    load8(vrow + d0, vf);
    load8(vrow + d1, vf + 8);
    const float mn = fmaxf(m, d);
    const float corr = __expf(m - mn), p = __expf(d - mn);
    l = l * corr + p;
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = acc[e] * corr + p * vf[e];
    m = mn;
  };
  int consumed = 0;
  for (int i = 0; i < nchunks; ++i) {
    const int c0 = beg + i * kChunk, n = min(kChunk, end - c0);
    if (!sm100::mbar_wait(&full_bar[i & 1], (i >> 1) & 1, a.timeout_ns, abort_flag)) {
      if (!*abort_flag) record_local_failure(a.err, a.err_host, kErrTimeout, kStageAttn, static_cast<uint32_t>(i));
      *abort_flag = 1;
    } else {
      consumed = i + 1;
    }
    const __nv_bfloat16* sk = kv_tile(i & 1, 0);
    const __nv_bfloat16* sv = kv_tile(i & 1, 1);
    if (owns_pos && warp == 0 && g == 0 && pos >= c0 && pos < c0 + n) {
      store8(kv_tile(i & 1, 0) + (pos - c0) * kHeadDim + d0, k_new);
      store8(kv_tile(i & 1, 0) + (pos - c0) * kHeadDim + d1, k_new + 8);
      store8(kv_tile(i & 1, 1) + (pos - c0) * kHeadDim + d0, v_new);
      store8(kv_tile(i & 1, 1) + (pos - c0) * kHeadDim + d1, v_new + 8);
    }
    __syncthreads();
    if (*abort_flag) break;
    if (warp < G) {
      // two positions of this group per iteration, both scores first; the
      // trip count is the same for every lane (the shuffles need the whole
      // warp), positions past the chunk are scored on a valid row and skipped
      for (int j0 = 0; j0 < n; j0 += 8) {
        const int ja = j0 + g, jb = j0 + 4 + g;
        float da = score(sk + min(ja, n - 1) * kHeadDim), db = score(sk + min(jb, n - 1) * kHeadDim);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          da += __shfl_xor_sync(0xffffffffu, da, o);
          db += __shfl_xor_sync(0xffffffffu, db, o);
        }
        if (ja < n) update(da, sv + ja * kHeadDim);
        if (jb < n) update(db, sv + jb * kHeadDim);
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (threadIdx.x == 0 && i + 2 < nchunks) issue(i + 2);
  }
  if (*abort_flag && threadIdx.x == 0) {
    // let copies still in flight land before the CTA's memory goes away
    volatile int never = 0;
    for (int i = consumed; i < issued; ++i) sm100::mbar_wait(&full_bar[i & 1], (i >> 1) & 1, a.timeout_ns, &never);
  }
  // merge the four groups' running states (xor 8, then 16)
  if (warp < G) {
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
      const float m_o = __shfl_xor_sync(0xffffffffu, m, o);
      const float l_o = __shfl_xor_sync(0xffffffffu, l, o);
      const float mn = fmaxf(m, m_o);
      const float w_me = m == -INFINITY ? 0.f : __expf(m - mn);
      const float w_o = m_o == -INFINITY ? 0.f : __expf(m_o - mn);
      l = l * w_me + l_o * w_o;
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] = acc[e] * w_me + __shfl_xor_sync(0xffffffffu, acc[e], o) * w_o;
      m = mn;
    }
  }
  if (warp < G && g == 0) {
    if (lane == 0) {
      s_m[warp] = m;
      s_l[warp] = l;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      s_o[warp][d0 + e] = acc[e];
      s_o[warp][d1 + e] = acc[8 + e];
    }
  }
  if (a.splits > 1) sm100::cluster_sync(); else __syncthreads();
  if (sp == 0 && warp < G) {
    // lane s reads split s's (m, l); weights exp(m_s - M), in split order
    const uint32_t m_addr = sm100::smem_u32(&s_m[warp]), l_addr = sm100::smem_u32(&s_l[warp]);
    const uint32_t o_addr = sm100::smem_u32(&s_o[warp][lane * 4]);
    float ms = -INFINITY, ls = 0.f;
    if (lane < a.splits) {
      ms = a.splits > 1 ? sm100::ld_dsmem_f32(sm100::dsmem_addr(m_addr, lane)) : s_m[warp];
      ls = a.splits > 1 ? sm100::ld_dsmem_f32(sm100::dsmem_addr(l_addr, lane)) : s_l[warp];
    }
    float M = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float wgt = ms == -INFINITY ? 0.f : __expf(ms - M);
    float den = wgt * ls;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    float num[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s2 = 0; s2 < a.splits; ++s2) {
      const float w = __shfl_sync(0xffffffffu, wgt, s2);
      if (w == 0.f) continue;
      const float4 o = a.splits > 1 ? sm100::ld_dsmem_f4(sm100::dsmem_addr(o_addr, s2))
                                    : *reinterpret_cast<const float4*>(&s_o[warp][lane * 4]);
      num[0] += w * o.x;
      num[1] += w * o.y;
      num[2] += w * o.z;
      num[3] += w * o.w;
    }
    const float inv = 1.f / den;
    const float r[4] = {num[0] * inv, num[1] * inv, num[2] * inv, num[3] * inv};
    *reinterpret_cast<uint2*>(a.out + (static_cast<int64_t>(b) * a.Hq + h) * kHeadDim + lane * 4) = pack4(r);
  }
  if (a.splits > 1) sm100::cluster_sync();  // CTA 0 has read every partial
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

namespace {

template <bool kRope>
void launch_attn(cudaStream_t s, const AttnArgs& a, int B) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    NAB_CUDA_CHECK(cudaFuncSetAttribute(k_attn<kRope>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    NAB_CUDA_CHECK(cudaFuncSetAttribute(k_attn<kRope>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
    attr_set[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.splits, B * a.Hkv);
  cfg.blockDim = dim3(32 * (a.Hq / a.Hkv));
  cfg.dynamicSmemBytes = kAttnSmem;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = a.splits;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn<kRope>, a);
  if (e != cudaSuccess) throw std::runtime_error(std::string("attention launch failed: ") + cudaGetErrorString(e));
}

void set_error_record(AttnArgs& a) {
  const KernelErrorRecord rec = kernel_error_record();
  a.err = rec.dev;
  a.err_host = rec.host;
  a.timeout_ns = kernel_timeout_ns();
}

void check_attn(int Hq, int Hkv, int splits) {
  if (Hkv < 1 || Hq % Hkv != 0 || Hq / Hkv > 8) throw std::invalid_argument("attention: need Hq / Hkv <= 8");
  if (splits < 1 || splits > kMaxAttnSplits) throw std::invalid_argument("attention: splits must be in [1, 16]");
}

}  // namespace

void decode_attention(cudaStream_t s, const void* q, const void* k_cache, const void* v_cache, const int* pos,
                      void* out, int B, int Hq, int Hkv, int Lmax, int splits) {
  check_attn(Hq, Hkv, splits);
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.pos = pos;
  a.k_cache = static_cast<__nv_bfloat16*>(const_cast<void*>(k_cache));
  a.v_cache = static_cast<__nv_bfloat16*>(const_cast<void*>(v_cache));
  a.out = static_cast<__nv_bfloat16*>(out);
  a.q_stride = Hq * kHeadDim;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.Lmax = Lmax;
  a.splits = splits;
  a.scale = 1.f / sqrtf(static_cast<float>(kHeadDim));
  set_error_record(a);
  launch_attn<false>(s, a, B);
}

void rope_attention(cudaStream_t s, const void* qkv, const float* cos_t, const float* sin_t, const int* pos,
                    void* k_cache, void* v_cache, void* out, int B, int Hq, int Hkv, int Lmax, int splits) {
  check_attn(Hq, Hkv, splits);
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(qkv);
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.pos = pos;
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.q_stride = (Hq + 2 * Hkv) * kHeadDim;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.Lmax = Lmax;
  a.splits = splits;
  a.scale = 1.f / sqrtf(static_cast<float>(kHeadDim));
  set_error_record(a);
  launch_attn<true>(s, a, B);
}

int attention_splits(int B, int Hkv, int context, int sms) {
  // about two CTAs per SM, at least 32 positions per split, one cluster of
  // a power-of-two size (those pack the GPCs without holes)
  const int want = std::max(1, (2 * sms) / std::max(1, B * Hkv));
  const int most = std::max(1, (context + 31) / 32);
  const int cap = std::min({want, most, kMaxAttnSplits});
  int sp = 1;
  while (sp * 2 <= cap) sp *= 2;
  return sp;
}

void silu_mul(cudaStream_t s, const void* gu, void* out, int B, int I) {
  const int64_t n = static_cast<int64_t>(B) * I;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
  k_silu_mul<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), B, I);
  check("silu_mul");
}

}  // namespace nab

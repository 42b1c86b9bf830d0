// GQA decode attention on the 5th-generation tensor cores (tcgen05 + TMEM),
// with the K/V chunks staged by TMA.
//
// One thread-block cluster of `splits` CTAs per (batch, kv head); CTA `sp`
// covers a contiguous range of positions in chunks of 128. Per chunk:
//   producer (warp 0, one thread)  TMA-loads the K and V chunk, 128 rows x
//       128 dims each, as two 64-dim boxes with 128-byte swizzle, into a
//       3-stage ring (mbarrier complete_tx);
//   scores   S^T[128 positions x 16 heads] = K . Q^T: 8 tcgen05.mma
//       (M=128, N=16, K=16), A = K (K-major), B = Q (the group's <= 8 query
//       heads, rows 8-15 zero), fp32 accumulator in TMEM columns 0-15 or
//       16-31 by chunk parity: the next chunk's scores are issued as soon as
//       this chunk's are read, so they run during this chunk's softmax;
//   softmax  4 warps read S from TMEM (one position per thread), mask
//       positions past the range, update the running max / sum per head
//       (warp shuffles + shared memory), write P (bf16) as a K-major tile;
//   values   O^T[128 dims x 16 heads] = V^T . P^T: 8 tcgen05.mma with A = V
//       read MN-major straight from the staged chunk (the cache is
//       [position][dim]), accumulator in TMEM columns 32-47; each thread (one
//       dim) rescales its running output and adds the chunk's.
// The splits' partial (max, sum, output) are combined by CTA 0 of the
// cluster over distributed shared memory: one launch, no scratch.
// kRope: q and the new k are rotated here from the qkv projection; the CTA
// whose range holds the current position writes k and v to the cache first
// (then a proxy fence, so the TMA load of that chunk sees them).
//
// Every mbarrier wait is bounded; one that runs out records into the
// device's kernel error record, the CTA stops issuing, waits (bounded) for
// its loads in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "nab_device.cuh"
#include "nab_driver.h"
#include "nab_kerr.h"
#include "nab_llama.h"
#include "nab_sm100.cuh"

namespace nab {

namespace {

constexpr int kD = 128;                  // head dim
constexpr int kTc = 128;                 // positions per chunk (the scores MMA's M)
constexpr int kStages = 3;               // K/V ring depth (3 x 64 KB: a split's first chunks load at once)
constexpr int kBox = kTc * 128;          // one TMA box: 128 rows x 64 dims (128 bytes)
constexpr int kStageBytes = 4 * kBox;    // K dims 0-63 | K 64-127 | V 0-63 | V 64-127
constexpr int kTileBytes = 16 * 128;     // Q or P: 16 rows x 64 elements, one swizzle tile
constexpr int kSmemTc = kStages * kStageBytes + 4 * kTileBytes + 1024;
constexpr int kThreadsTc = 160;          // warp 0: TMA producer; warps 1-4: MMA, softmax, output
constexpr int kMaxSplitsTc = 16;
constexpr uint32_t kTmemCols = 64;       // S in columns 0-15 / 16-31 (chunk parity), O in 32-47

struct AttnTcArgs {
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
  ErrorState* err;
  uint32_t* err_host;
  uint64_t timeout_ns;
};

NAB_DINLINE void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
NAB_DINLINE void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
NAB_DINLINE void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Byte offset of element (row, col) of a 64-column bf16 tile with 128-byte
// swizzle (rows of 128 bytes, 16-byte chunks permuted by row % 8): the
// layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B and tcgen05 reads.
NAB_DINLINE uint32_t sw128(int row, int col) {
  return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) + (col & 7) * 2);
}

// Descriptor of an MN-major tile with 128-byte swizzle: 64 MN-elements per
// 128-byte row, consecutive K in consecutive rows (8-row groups `sbo` bytes
// apart), the next 64 MN-elements `lbo` bytes further.
NAB_DINLINE uint64_t smem_desc_mn_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // version
  d |= static_cast<uint64_t>(2u) << 61;  // swizzle 128 B
  return d;
}

NAB_DINLINE float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
NAB_DINLINE float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <bool kRope>
__global__ void __launch_bounds__(kThreadsTc, 1)
    k_attn_tc(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
              const __grid_constant__ AttnTcArgs a) {
  extern __shared__ uint8_t attn_tc_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_tc_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                          // [stage][K0 | K1 | V0 | V1]
  uint8_t* qs = smem + kStages * kStageBytes;    // Q tiles: dims 0-63 | dims 64-127
  uint8_t* ps = qs + 2 * kTileBytes;             // P tiles: positions 0-63 | 64-127
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ __align__(8) uint64_t mma_bar;   // scores of a chunk done (one phase per chunk)
  __shared__ __align__(8) uint64_t out_bar;   // output MMAs of a chunk done
  __shared__ __align__(8) uint64_t kvnew_bar;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ float s_red[4][8];
  __shared__ float s_m[8], s_l[8];
  __shared__ __align__(16) float s_o[8][kD];
  volatile int* abort_flag = &s_abort;

  const int sp = blockIdx.x, b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ct = threadIdx.x - 32;  // compute thread 0..127 (warps 1-4)

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    sm100::mbar_init(&mma_bar, 1);
    sm100::mbar_init(&out_bar, 1);
    sm100::mbar_init(&kvnew_bar, 1);
    sm100::fence_barrier_init();
    s_abort = 0;
    sm100::prefetch_tensormap(&tk);
    sm100::prefetch_tensormap(&tv);
  }
  if (warp == 1) {
    sm100::tmem_alloc(&s_tmem, kTmemCols);
    sm100::tmem_relinquish();
  }
  // zero the Q and P tiles (rows of heads past the group stay zero)
  for (int i = threadIdx.x; i < 4 * kTileBytes / 16; i += kThreadsTc)
    reinterpret_cast<uint4*>(qs)[i] = make_uint4(0u, 0u, 0u, 0u);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = s_tmem;

  sm100::griddep_wait();  // inputs come from the kernel before (programmatic launch)
  pdl_trigger();
  const int pos = *a.pos;
  const int L = pos + 1;
  const int per = (L + a.splits - 1) / a.splits;
  const int beg = sp * per, end = min(L, beg + per);
  const int nchunks = end > beg ? (end - beg + kTc - 1) / kTc : 0;
  const int row0 = (b * a.Hkv + kvh) * a.Lmax;  // first cache row of this (batch, kv head)
  const bool owns_pos = kRope && beg <= pos && pos < end;
  const __nv_bfloat16* qrow = a.q + static_cast<int64_t>(b) * a.q_stride;

  auto fail = [&](uint32_t observed) {
    if (!*abort_flag) record_local_failure(a.err, a.err_host, kErrTimeout, kStageAttn, observed);
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nchunks; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !sm100::mbar_wait(&empty_bar[s], ((i / kStages) - 1) & 1, a.timeout_ns, abort_flag)) {
          fail(static_cast<uint32_t>(i));
          break;
        }
        const int c0 = beg + i * kTc;
        // the chunk holding the new position: its k and v must be in the cache
        if (owns_pos && c0 <= pos && pos < c0 + kTc && !sm100::mbar_wait(&kvnew_bar, 0, a.timeout_ns, abort_flag)) {
          fail(static_cast<uint32_t>(i));
          break;
        }
        if (*abort_flag) break;
        uint8_t* st = ring + s * kStageBytes;
        sm100::mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
        sm100::tma_load_2d(st, &tk, 0, row0 + c0, &full_bar[s]);
        sm100::tma_load_2d(st + kBox, &tk, 64, row0 + c0, &full_bar[s]);
        sm100::tma_load_2d(st + 2 * kBox, &tv, 0, row0 + c0, &full_bar[s]);
        sm100::tma_load_2d(st + 3 * kBox, &tv, 64, row0 + c0, &full_bar[s]);
        ++issued;
      }
      if (*abort_flag) {
        // let the loads already issued land before the CTA's memory goes away
        volatile int never = 0;
        for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
          sm100::mbar_wait(&full_bar[i % kStages], (i / kStages) & 1, a.timeout_ns, &never);
      }
    }
  } else {
    // ------------------------------------------- prologue: Q, new k and v
    {
      // thread -> (head h = ct / 8, dims [8c, 8c + 8) and [64 + 8c, 64 + 8c + 8))
      const int h = ct >> 3, c = ct & 7;
      if (h < G) {
        const __nv_bfloat16* src = qrow + static_cast<int64_t>(kvh * G + h) * kD;
        const uint4 lo = *reinterpret_cast<const uint4*>(src + 8 * c);
        const uint4 hi = *reinterpret_cast<const uint4*>(src + 64 + 8 * c);
        uint4 olo = lo, ohi = hi;
        if (kRope) {
          const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w}, wh[4] = {hi.x, hi.y, hi.z, hi.w};
          uint32_t rl[4], rh[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float x1[2] = {bf_lo(wl[k]), bf_hi(wl[k])}, x2[2] = {bf_lo(wh[k]), bf_hi(wh[k])};
            float y1[2], y2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int d = 8 * c + 2 * k + e;
              const float cs = a.cos_t[pos * (kD / 2) + d], sn = a.sin_t[pos * (kD / 2) + d];
              y1[e] = x1[e] * cs - x2[e] * sn;
              y2[e] = x2[e] * cs + x1[e] * sn;
            }
            rl[k] = pack_bf16x2(y1[0], y1[1]);
            rh[k] = pack_bf16x2(y2[0], y2[1]);
          }
          olo = make_uint4(rl[0], rl[1], rl[2], rl[3]);
          ohi = make_uint4(rh[0], rh[1], rh[2], rh[3]);
        }
        *reinterpret_cast<uint4*>(qs + sw128(h, 8 * c)) = olo;
        *reinterpret_cast<uint4*>(qs + kTileBytes + sw128(h, 8 * c)) = ohi;
      }
      if (owns_pos && ct < 16) {
        // threads 0-7: k (rotated), 8-15: v, dims [8c, 8c + 8) and [64 + 8c, ...)
        const int cc = ct & 7;
        const bool is_k = ct < 8;
        const __nv_bfloat16* src = qrow + static_cast<int64_t>(a.Hq + (is_k ? 0 : a.Hkv) + kvh) * kD;
        uint4 lo = *reinterpret_cast<const uint4*>(src + 8 * cc);
        uint4 hi = *reinterpret_cast<const uint4*>(src + 64 + 8 * cc);
        if (is_k) {
          const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w}, wh[4] = {hi.x, hi.y, hi.z, hi.w};
          uint32_t rl[4], rh[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float x1[2] = {bf_lo(wl[k]), bf_hi(wl[k])}, x2[2] = {bf_lo(wh[k]), bf_hi(wh[k])};
            float y1[2], y2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int d = 8 * cc + 2 * k + e;
              const float cs = a.cos_t[pos * (kD / 2) + d], sn = a.sin_t[pos * (kD / 2) + d];
              y1[e] = x1[e] * cs - x2[e] * sn;
              y2[e] = x2[e] * cs + x1[e] * sn;
            }
            rl[k] = pack_bf16x2(y1[0], y1[1]);
            rh[k] = pack_bf16x2(y2[0], y2[1]);
          }
          lo = make_uint4(rl[0], rl[1], rl[2], rl[3]);
          hi = make_uint4(rh[0], rh[1], rh[2], rh[3]);
        }
        __nv_bfloat16* dst = (is_k ? a.k_cache : a.v_cache) + (static_cast<int64_t>(row0) + pos) * kD;
        *reinterpret_cast<uint4*>(dst + 8 * cc) = lo;
        *reinterpret_cast<uint4*>(dst + 64 + 8 * cc) = hi;
        fence_async_global();  // the TMA load of this row must see the stores
      }
      fence_async_shared();    // Q tile visible to the tensor core
      sm100::tc_fence_before();
      named_sync(1, 128);
      sm100::tc_fence_after();
      if (owns_pos && ct == 0) sm100::mbar_arrive(&kvnew_bar);
    }

    // ----------------------------------------------------------- chunks
    // The compute threads leave the loop together: the barrier ORs every
    // thread's view of the abort flag (the producer may set it at any time).
    auto agreed_abort = [&]() -> bool { return named_barrier_or(1, 128, *abort_flag != 0); };
    const int q4 = warp & 3;                 // TMEM lane quarter of this warp
    const int row = q4 * 32 + lane;          // position (scores) / dim (output)
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    constexpr uint32_t idesc_s = sm100::idesc_bf16_f32(kTc, 16);
    constexpr uint32_t idesc_o = sm100::idesc_bf16_f32(kD, 16) | (1u << 15);  // A (V) MN-major
    float m[8], l[8], acc[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.f;
      acc[h] = 0.f;
    }
    // S^T = K . Q^T of chunk j into TMEM columns 16 (j & 1) .. + 15 (thread 0
    // of the group, once the chunk's stage landed), committed to mma_bar: one
    // phase per chunk. Waits on this CTA's own MMAs use `never` so that no MMA
    // is still in flight when the CTA leaves.
    volatile int never = 0;
    auto scores_mma = [&](int j) {
      sm100::tc_fence_after();
      const uint32_t ka = sm100::smem_u32(ring + (j % kStages) * kStageBytes), qa = sm100::smem_u32(qs);
#pragma unroll
      for (int k = 0; k < kD / 16; ++k) {
        const uint32_t off = (k >> 2) * kBox + (k & 3) * 32;
        const uint32_t qoff = (k >> 2) * kTileBytes + (k & 3) * 32;
        sm100::mma_bf16(tmem + 16 * (j & 1), sm100::smem_desc_k_sw128(ka + off), sm100::smem_desc_k_sw128(qa + qoff),
                        idesc_s, k != 0);
      }
      sm100::mma_commit(&mma_bar);
    };
    // blocking: waits (bounded) for the stage; false, after recording, if it never landed
    auto issue_scores = [&](int j) -> bool {
      if (!sm100::mbar_wait(&full_bar[j % kStages], (j / kStages) & 1, a.timeout_ns, abort_flag)) {
        fail(j);
        return false;
      }
      scores_mma(j);
      return true;
    };
    bool pending = false;  // thread 0: the scores of chunk i were issued
    for (int i = 0; i < nchunks; ++i) {
      const int s = i % kStages;
      uint8_t* st = ring + s * kStageBytes;
      const int c0 = beg + i * kTc, n = min(kTc, end - c0);
      // scores of chunk i (phase i of mma_bar), issued now unless issued early
      if (ct == 0) {
        if (!pending && !*abort_flag) pending = issue_scores(i);
        if (pending && !sm100::mbar_wait(&mma_bar, i & 1, a.timeout_ns, &never)) fail(i);
        pending = false;
        sm100::tc_fence_before();
      }
      if (agreed_abort()) break;
      sm100::tc_fence_after();
      uint32_t r[16];
      sm100::tmem_ld16(tmem + t_lane + 16 * (i & 1), r);
      sm100::tmem_wait_ld();
      float p[8];
      const bool valid = row < n;
#pragma unroll
      for (int h = 0; h < 8; ++h) p[h] = (valid && h < G) ? __uint_as_float(r[h]) * a.scale : -INFINITY;
      if (n < kTc) {
        // rows past the range: P is zero there, and V must not hold NaN
        for (int rr = n + (ct >> 4); rr < kTc; rr += 8) {
          reinterpret_cast<uint4*>(st + 2 * kBox + rr * 128)[ct & 7] = make_uint4(0u, 0u, 0u, 0u);
          reinterpret_cast<uint4*>(st + 3 * kBox + rr * 128)[ct & 7] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      // chunk max per head
      float mx[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        float v = p[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        mx[h] = v;
      }
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < 8; ++h) s_red[q4][h] = mx[h];
      }
      sm100::tc_fence_before();
      named_sync(1, 128);  // every thread has read S(i): its TMEM buffer is free
      // scores of chunk i + 1 run on the tensor cores during this softmax, if
      // its stage has landed already (otherwise at the top of the next chunk)
      if (ct == 0 && i + 1 < nchunks && !*abort_flag &&
          sm100::mbar_try_wait(&full_bar[(i + 1) % kStages], ((i + 1) / kStages) & 1)) {
        scores_mma(i + 1);
        pending = true;
      }
      float alpha[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const float cm = fmaxf(fmaxf(s_red[0][h], s_red[1][h]), fmaxf(s_red[2][h], s_red[3][h]));
        const float mn = fmaxf(m[h], cm);
        alpha[h] = m[h] == -INFINITY ? 0.f : __expf(m[h] - mn);
        p[h] = p[h] == -INFINITY ? 0.f : __expf(p[h] - mn);
        m[h] = mn;
      }
      // P row (this position) of every head, bf16, into the K-major P tiles;
      // the sums use the rounded values the MMA multiplies
      {
        const int t = row >> 6, col = row & 63;
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const __nv_bfloat16 pb = __float2bfloat16_rn(p[h]);
          p[h] = __bfloat162float(pb);
          *reinterpret_cast<__nv_bfloat16*>(ps + t * kTileBytes + sw128(h, col)) = pb;
        }
      }
      float sm[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        float v = p[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        sm[h] = v;
      }
      fence_async_shared();  // P and the zeroed V rows, before the tensor core reads them
      named_sync(1, 128);    // every thread has read s_red (max) and written P
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < 8; ++h) s_red[q4][h] = sm[h];
      }
      // O^T = V^T . P^T (the commit also covers the scores issued above)
      if (ct == 0) {
        sm100::tc_fence_after();
        const uint32_t va = sm100::smem_u32(st + 2 * kBox), pa = sm100::smem_u32(ps);
#pragma unroll
        for (int j = 0; j < kTc / 16; ++j) {
          const uint32_t poff = (j >> 2) * kTileBytes + (j & 3) * 32;
          sm100::mma_bf16(tmem + 32, smem_desc_mn_sw128(va + j * 16 * 128, kBox, 1024),
                          sm100::smem_desc_k_sw128(pa + poff), idesc_o, j != 0);
        }
        sm100::mma_commit(&out_bar);
        sm100::mma_commit(&empty_bar[s]);  // the stage is free once these MMAs completed
        if (!sm100::mbar_wait(&out_bar, i & 1, a.timeout_ns, &never)) fail(i);
        sm100::tc_fence_before();
      }
      if (agreed_abort()) break;
      sm100::tc_fence_after();
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const float cs = (s_red[0][h] + s_red[1][h]) + (s_red[2][h] + s_red[3][h]);
        l[h] = l[h] * alpha[h] + cs;
      }
      sm100::tmem_ld16(tmem + t_lane + 32, r);
      sm100::tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < 8; ++h) acc[h] = acc[h] * alpha[h] + __uint_as_float(r[h]);
      sm100::tc_fence_before();
      named_sync(1, 128);  // s_red, P and the output columns free for the next chunk
    }
    // this split's partial: (max, sum) per head, unnormalised output per dim
    if (ct < 8) {
      s_m[ct] = m[ct];
      s_l[ct] = l[ct];
    }
#pragma unroll
    for (int h = 0; h < 8; ++h)
      if (h < G) s_o[h][row] = acc[h];
  }
  if (a.splits > 1) sm100::cluster_sync(); else __syncthreads();
  if (sp == 0 && !*abort_flag) {
    // warp w combines heads w, w + 5, ...: lane s reads split s's (m, l)
    for (int h = warp; h < G; h += kThreadsTc / 32) {
      const uint32_t m_addr = sm100::smem_u32(&s_m[h]), l_addr = sm100::smem_u32(&s_l[h]);
      const uint32_t o_addr = sm100::smem_u32(&s_o[h][lane * 4]);
      float ms = -INFINITY, ls = 0.f;
      if (lane < a.splits) {
        ms = a.splits > 1 ? sm100::ld_dsmem_f32(sm100::dsmem_addr(m_addr, lane)) : s_m[h];
        ls = a.splits > 1 ? sm100::ld_dsmem_f32(sm100::dsmem_addr(l_addr, lane)) : s_l[h];
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
                                      : *reinterpret_cast<const float4*>(&s_o[h][lane * 4]);
        num[0] += w * o.x;
        num[1] += w * o.y;
        num[2] += w * o.z;
        num[3] += w * o.w;
      }
      const float inv = 1.f / den;
      uint2 packed;
      packed.x = pack_bf16x2(num[0] * inv, num[1] * inv);
      packed.y = pack_bf16x2(num[2] * inv, num[3] * inv);
      *reinterpret_cast<uint2*>(a.out + (static_cast<int64_t>(b) * a.Hq + kvh * G + h) * kD + lane * 4) = packed;
    }
  }
  if (a.splits > 1) sm100::cluster_sync();  // CTA 0 has read every partial
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------ host side --
using PFN_Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The cache [rows, 128] bf16 with a box of 128 rows x 64 dims, 128-byte swizzle.
CUtensorMap cache_map(const void* ptr, int64_t rows) {
  static std::mutex mu;
  static std::unordered_map<std::string, CUtensorMap> cache;
  char key[64];
  std::snprintf(key, sizeof(key), "%p/%lld", ptr, static_cast<long long>(rows));
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) throw std::invalid_argument("attention: KV cache must be 16-byte aligned");
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD) * 2};
  const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(kTc)};
  const cuuint32_t estr[2] = {1, 1};
  NAB_CU_CHECK(driver_fn<PFN_Encode>("cuTensorMapEncodeTiled")(
      &m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  return m;
}

template <bool kRope>
void launch_tc(cudaStream_t s, const AttnTcArgs& a, int B) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    NAB_CUDA_CHECK(cudaFuncSetAttribute(k_attn_tc<kRope>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    NAB_CUDA_CHECK(cudaFuncSetAttribute(k_attn_tc<kRope>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc));
    attr_set[dev & 63] = true;
  }
  const int64_t rows = static_cast<int64_t>(B) * a.Hkv * a.Lmax;
  const CUtensorMap tk = cache_map(a.k_cache, rows), tv = cache_map(a.v_cache, rows);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.splits, B * a.Hkv);
  cfg.blockDim = dim3(kThreadsTc);
  cfg.dynamicSmemBytes = kSmemTc;
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn_tc<kRope>, tk, tv, a);
  if (e != cudaSuccess) throw std::runtime_error(std::string("attention launch failed: ") + cudaGetErrorString(e));
}

AttnTcArgs make_args(int Hq, int Hkv, int Lmax, int splits) {
  if (Hkv < 1 || Hq % Hkv != 0 || Hq / Hkv > 8) throw std::invalid_argument("attention: need Hq / Hkv <= 8");
  if (splits < 1 || splits > kMaxSplitsTc) throw std::invalid_argument("attention: splits must be in [1, 16]");
  if (Lmax < 1) throw std::invalid_argument("attention: bad cache length");
  AttnTcArgs a{};
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.Lmax = Lmax;
  a.splits = splits;
  a.scale = 1.f / std::sqrt(static_cast<float>(kD));
  const KernelErrorRecord rec = kernel_error_record();
  a.err = rec.dev;
  a.err_host = rec.host;
  a.timeout_ns = kernel_timeout_ns();
  return a;
}

}  // namespace

void decode_attention_tc(cudaStream_t s, const void* q, const void* k_cache, const void* v_cache, const int* pos,
                         void* out, int B, int Hq, int Hkv, int Lmax, int splits) {
  AttnTcArgs a = make_args(Hq, Hkv, Lmax, splits);
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.pos = pos;
  a.k_cache = static_cast<__nv_bfloat16*>(const_cast<void*>(k_cache));
  a.v_cache = static_cast<__nv_bfloat16*>(const_cast<void*>(v_cache));
  a.out = static_cast<__nv_bfloat16*>(out);
  a.q_stride = Hq * kD;
  launch_tc<false>(s, a, B);
}

void rope_attention_tc(cudaStream_t s, const void* qkv, const float* cos_t, const float* sin_t, const int* pos,
                       void* k_cache, void* v_cache, void* out, int B, int Hq, int Hkv, int Lmax, int splits) {
  AttnTcArgs a = make_args(Hq, Hkv, Lmax, splits);
  a.q = static_cast<const __nv_bfloat16*>(qkv);
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.pos = pos;
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.q_stride = (Hq + 2 * Hkv) * kD;
  launch_tc<true>(s, a, B);
}

int attention_splits_tc(int B, int Hkv, int context, int sms) {
  // one CTA per SM (137 KB of shared memory each): the largest power of two
  // that keeps every CTA of the launch resident, with at least one chunk of
  // 128 positions per split
  const int groups = std::max(1, B * Hkv);
  const int fit = std::max(1, sms / groups);
  const int most = std::max(1, (context + kTc - 1) / kTc);
  const int cap = std::min({fit, most, kMaxSplitsTc});
  int sp = 1;
  while (sp * 2 <= cap) sp *= 2;
  return sp;
}

}  // namespace nab

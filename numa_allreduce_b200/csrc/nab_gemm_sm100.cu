// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA) for the
// tensor-parallel projections, and its fusion with the allreduce.
//
//   y[T, N] = x[T, K] . Wt[N, K]^T        (Wt: the weight stored K-major)
//
// Decode-time T is tiny, so the kernel computes the transposed product: each
// CTA owns 128 output features (rows of Wt, the MMA's M) and up to 256 tokens
// (the MMA's N), accumulating over K in TMEM. Roles per CTA (6 warps):
//   warp 0   TMA producer: Wt and x tiles into a ring of shared-memory stages
//            (128-byte swizzle, K-major), completion counted on mbarriers;
//   warp 1   allocates TMEM, issues tcgen05.mma (M=128, N=BN, K=16) and
//            commits each stage back to the producer;
//   warps 2-5  epilogue: tcgen05.ld the accumulator, convert to bf16, stage
//            the tile in shared memory as [token][feature] and write it out.
// Split-K (grid dimension `splits`) gives small-N layers enough CTAs: each
// split writes an fp32 partial and a second kernel adds them in split order.
//
// Fused with the allreduce (no counterpart in the reference, which has no
// fused ops): the epilogue stores the bf16 partial tile straight into every
// rank's one-shot slot over NVLink (its own slot included), then exchanges a
// per-tile flag with the same CTA on every peer. When the kernel ends every
// peer's partials of every tile are in local memory, and a second kernel adds
// them in rank order with the residual and applies RMSNorm.
//
// Every mbarrier and flag wait is bounded; on expiry the CTA stops issuing,
// waits (bounded) for its TMA loads in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "nab_comm.h"
#include "nab_driver.h"
#include "nab_fused.h"
#include "nab_gemm.h"
#include "nab_proto.cuh"
#include "nab_sm100.cuh"

namespace nab {

namespace {

constexpr int kGemmThreads = 192;
constexpr int kBM = 128;
constexpr int kBK = 64;  // 128 bytes of bf16: one swizzle atom row
constexpr int kABytes = kBM * kBK * 2;

struct GemmArgs {
  int M;          // output features (rows of Wt), multiple of 128
  int K;          // multiple of 64
  int T;          // tokens
  int m_tiles;
  int n_tiles;
  int splits;
  int kb_per_split;
  int fused;
  __nv_bfloat16* out;  // [T, M] bf16 (splits == 1, not fused)
  float* partial;      // [splits, T, M] fp32 (splits > 1)
  // fused allreduce epilogue
  char* wsp[kMaxRanks];
  int rank;
  int ws;
  int64_t slot_off;    // fused one-shot slots: [2 parities][ws][slot_bytes]
  int64_t slot_bytes;
  ErrorState* err;
  uint32_t* err_host;
  uint64_t timeout_ns;
};

template <int BN>
struct GemmCfg {
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN <= 64 ? 8 : (BN == 128 ? 6 : 4);
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024;  // + alignment slack
};

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ GemmArgs g) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t accum_bar;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int m_tile = tile % g.m_tiles;
  const int rest = tile / g.m_tiles;
  const int n_tile = rest % g.n_tiles;
  const int split = rest / g.n_tiles;
  const int m0 = m_tile * kBM;
  const int t0 = n_tile * BN;
  const int kb0 = split * g.kb_per_split;
  const int kb1 = min(g.K / kBK, kb0 + g.kb_per_split);
  const int nkb = kb1 - kb0;

  uint32_t epoch = 0;
  if (g.fused) epoch = begin_call(g.wsp, g.rank);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    sm100::mbar_init(&accum_bar, 1);
    sm100::fence_barrier_init();
    s_abort = 0;
    sm100::prefetch_tensormap(&tmA);
    sm100::prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    sm100::tmem_alloc(&s_tmem, Cfg::kTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = s_tmem;

  auto fail = [&](uint32_t stage) {
    if (g.err != nullptr && !*abort_flag) {
      WaitCtx w = make_wait(g.err, g.err_host, g.timeout_ns, g.wsp, g.rank, epoch);
      if (g.fused) record_failure(w, kErrTimeout, 0xffffffffu, stage, 0);
    }
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (i >= S && !sm100::mbar_wait(&empty_bar[s], ((i / S) - 1) & 1, g.timeout_ns, abort_flag)) {
          fail(kStageGemmAR);
          break;
        }
        if (*abort_flag) break;
        uint8_t* sa = smem + s * Cfg::kStageBytes;
        sm100::mbar_arrive_expect_tx(&full_bar[s], Cfg::kStageBytes);
        sm100::tma_load_2d(sa, &tmA, (kb0 + i) * kBK, m0, &full_bar[s]);
        sm100::tma_load_2d(sa + kABytes, &tmB, (kb0 + i) * kBK, t0, &full_bar[s]);
        ++issued;
      }
      if (*abort_flag) {
        // let the loads already issued land before the CTA's memory goes away
        volatile int never = 0;
        for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
          sm100::mbar_wait(&full_bar[i % S], (i / S) & 1, g.timeout_ns, &never);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(kBM, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (!sm100::mbar_wait(&full_bar[s], (i / S) & 1, g.timeout_ns, abort_flag)) {
          fail(kStageGemmAR);
          break;
        }
        sm100::tc_fence_after();
        const uint32_t a = sm100::smem_u32(smem + s * Cfg::kStageBytes);
        const uint32_t b = a + kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)
          sm100::mma_bf16(tmem, sm100::smem_desc_k_sw128(a + k * 32), sm100::smem_desc_k_sw128(b + k * 32), idesc,
                          (i | k) != 0);
        sm100::mma_commit(&empty_bar[s]);
      }
      sm100::mma_commit(&accum_bar);  // fires once every MMA above completed
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int q = warp & 3;        // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;  // feature within the tile
    const int et = threadIdx.x - 64;
    if (!sm100::mbar_wait(&accum_bar, 0, g.timeout_ns, abort_flag)) fail(kStageGemmAR);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const bool ok = !*abort_flag;  // uniform over the epilogue warps
    sm100::tc_fence_after();
    const int rows = min(BN, g.T - t0);  // valid tokens of this tile
    if (ok && nkb > 0) {
      if (g.splits > 1 && !g.fused) {
        // fp32 partial: [split][t][m]
        float* dstp = g.partial + (static_cast<int64_t>(split) * g.T) * g.M + m0 + row;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          sm100::tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < rows) dstp[static_cast<int64_t>(t0 + c0 + j) * g.M] = __uint_as_float(r[j]);
        }
      } else if (g.splits > 1) {
        // fused split-K: stage [token][feature] fp32 and store it into every
        // rank's slot as [split][t][m] fp32
        float* st = reinterpret_cast<float*>(smem);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          sm100::tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) st[(c0 + j) * kBM + row] = __uint_as_float(r[j]);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const uint4* st4 = reinterpret_cast<const uint4*>(st);
        const int nvec = rows * (kBM / 4);  // 32 x 16 B per token row
        const int parity = epoch & 1;
        for (int idx = et; idx < nvec; idx += 128) {
          const int t = idx >> 5, v = idx & 31;
          const uint4 val = st4[idx];
          const int64_t off = ((static_cast<int64_t>(split) * g.T + t0 + t) * g.M + m0) * 4;
          for (int k = 0; k < g.ws; ++k) {
            const int dst = (g.rank + k) % g.ws;
            char* slot = g.wsp[dst] + g.slot_off + (static_cast<int64_t>(parity) * g.ws + g.rank) * g.slot_bytes;
            reinterpret_cast<uint4*>(slot + off)[v] = val;
          }
        }
      } else {
        // stage [token][feature] bf16 in the (now idle) pipeline memory
        __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(smem);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          sm100::tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) st[(c0 + j) * kBM + row] = __float2bfloat16_rn(__uint_as_float(r[j]));
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const uint4* st4 = reinterpret_cast<const uint4*>(st);
        const int nvec = rows * (kBM / 8);  // 16 x 16 B per token row
        if (!g.fused) {
          for (int idx = et; idx < nvec; idx += 128) {
            const int t = idx >> 4, v = idx & 15;
            reinterpret_cast<uint4*>(g.out + static_cast<int64_t>(t0 + t) * g.M + m0)[v] = st4[idx];
          }
        } else {
          const int parity = epoch & 1;
          for (int idx = et; idx < nvec; idx += 128) {
            const int t = idx >> 4, v = idx & 15;
            const uint4 val = st4[idx];
            const int64_t off = (static_cast<int64_t>(t0 + t) * g.M + m0) * 2;
            for (int k = 0; k < g.ws; ++k) {
              const int dst = (g.rank + k) % g.ws;  // stagger the peers
              char* slot = g.wsp[dst] + g.slot_off + (static_cast<int64_t>(parity) * g.ws + g.rank) * g.slot_bytes;
              reinterpret_cast<uint4*>(slot + off)[v] = val;
            }
          }
        }
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (g.fused && !*abort_flag) {
      // exchange this tile's flag with the same CTA on every peer
      if (et < g.ws - 1) {
        const int peer = (g.rank + 1 + et) % g.ws;
        const uint64_t seq = make_seq(epoch, 0);
        st_release_sys(&pad_at(g.wsp, peer)->flags[kFlagGemm].v[tile][g.rank], seq);
        WaitCtx w = make_wait(g.err, g.err_host, g.timeout_ns, g.wsp, g.rank, epoch);
        if (!wait_geq(&pad_at(g.wsp, g.rank)->flags[kFlagGemm].v[tile][peer], seq, w, peer, kStageGemmAR))
          *abort_flag = 1;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (g.fused) end_call(g.wsp, g.rank, epoch);
}

// Adds the split-K partials in split order and rounds to bf16.
__global__ void k_splitk_reduce(const float* __restrict__ partial, __nv_bfloat16* __restrict__ out, int splits,
                                int64_t n4) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 a = reinterpret_cast<const float4*>(partial)[i];
    for (int s = 1; s < splits; ++s) {
      const float4 b = reinterpret_cast<const float4*>(partial + s * n4 * 4)[i];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
    uint2 v;
    v.x = *reinterpret_cast<uint32_t*>(&lo);
    v.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(out)[i] = v;
  }
}

// ------------------------------------------------------------ tensor maps --
using PFN_Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// K-major bf16 matrix [rows, K] with a box of [box_rows, 64] and 128-byte swizzle.
CUtensorMap make_map(const void* ptr, int64_t rows, int64_t K, int box_rows) {
  static std::mutex mu;
  static std::unordered_map<std::string, CUtensorMap> cache;
  char key[96];
  std::snprintf(key, sizeof(key), "%p/%lld/%lld/%d", ptr, static_cast<long long>(rows), static_cast<long long>(K),
                box_rows);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) throw std::invalid_argument("GEMM operands must be 16-byte aligned");
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  NAB_CU_CHECK(driver_fn<PFN_Encode>("cuTensorMapEncodeTiled")(
      &m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  return m;
}

int pick_bn(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}

template <int BN>
void launch_bn(const CUtensorMap& a, const CUtensorMap& b, const GemmArgs& g, int grid, cudaStream_t s) {
  using Cfg = GemmCfg<BN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    NAB_CUDA_CHECK(cudaFuncSetAttribute(k_gemm_bf16<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem));
    attr_set[dev & 63] = true;
  }
  k_gemm_bf16<BN><<<grid, kGemmThreads, Cfg::kSmem, s>>>(a, b, g);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("GEMM launch failed: ") + cudaGetErrorString(e));
}

void launch(const void* wt, const void* x, const GemmArgs& g, int bn, cudaStream_t s) {
  const CUtensorMap a = make_map(wt, g.M, g.K, kBM);
  const CUtensorMap b = make_map(x, g.T, g.K, bn);
  const int grid = g.m_tiles * g.n_tiles * g.splits;
  switch (bn) {
    case 16: launch_bn<16>(a, b, g, grid, s); break;
    case 32: launch_bn<32>(a, b, g, grid, s); break;
    case 64: launch_bn<64>(a, b, g, grid, s); break;
    case 128: launch_bn<128>(a, b, g, grid, s); break;
    default: launch_bn<256>(a, b, g, grid, s); break;
  }
}

void check_shape(int T, int N, int K) {
  if (T < 1 || N < kBM || N % kBM != 0 || K < kBK || K % kBK != 0)
    throw std::invalid_argument("GEMM needs T >= 1, N a multiple of 128 and K a multiple of 64");
}

}  // namespace

int gemm_splits_for(int T, int N, int K, int sms) {
  const int bn = pick_bn(T);
  const int tiles = (N / kBM) * ((T + bn - 1) / bn);
  const int kb = K / kBK;
  int splits = 1;
  // enough CTAs to stream the weight from every SM, at least 8 k-blocks each
  while (tiles * splits * 2 <= sms && kb / (splits * 2) >= 8) splits *= 2;
  return splits;
}

void gemm_bf16(cudaStream_t s, const void* wt, const void* x, void* y, int T, int N, int K, float* splitk_ws,
               int64_t splitk_ws_floats, int splits) {
  check_shape(T, N, K);
  GemmArgs g{};
  const int bn = pick_bn(T);
  g.M = N;
  g.K = K;
  g.T = T;
  g.m_tiles = N / kBM;
  g.n_tiles = (T + bn - 1) / bn;
  g.splits = std::max(1, splits);
  g.kb_per_split = (K / kBK + g.splits - 1) / g.splits;
  g.splits = (K / kBK + g.kb_per_split - 1) / g.kb_per_split;
  g.out = static_cast<__nv_bfloat16*>(y);
  g.timeout_ns = 2000000000ull;
  if (g.splits > 1) {
    const int64_t need = static_cast<int64_t>(g.splits) * T * N;
    if (splitk_ws == nullptr || splitk_ws_floats < need)
      throw std::invalid_argument("split-K GEMM needs a workspace of splits * T * N floats");
    g.partial = splitk_ws;
  }
  launch(wt, x, g, bn, s);
  if (g.splits > 1) {
    const int64_t n4 = static_cast<int64_t>(T) * N / 4;
    const int blocks = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, 148 * 4));
    k_splitk_reduce<<<blocks, 256, 0, s>>>(splitk_ws, static_cast<__nv_bfloat16*>(y), g.splits, n4);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("split-K reduce failed: ") + cudaGetErrorString(e));
  }
}

int gemm_allreduce_rmsnorm(Communicator& c, cudaStream_t s, const void* wt, const void* x, void* residual,
                           const void* weight, void* out, int T, int N, int K, float eps, int splits) {
  check_shape(T, N, K);
  const Layout& L = c.layout();
  if (c.world_size() == 1) throw std::invalid_argument("GEMM+allreduce needs a world size of at least 2");
  const int bn = pick_bn(T);
  GemmArgs g{};
  g.M = N;
  g.K = K;
  g.T = T;
  g.m_tiles = N / kBM;
  g.n_tiles = (T + bn - 1) / bn;
  if (splits <= 0) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    splits = gemm_splits_for(T, N, K, sms);
  }
  // one split: bf16 partials; several: fp32 partials, one per split. Fewer
  // splits until the partials fit the slot.
  auto need = [&](int sp) {
    return sp > 1 ? static_cast<int64_t>(sp) * T * N * 4 : static_cast<int64_t>(T) * N * 2;
  };
  while (splits > 1 && need(splits) > L.fused_bytes) splits /= 2;
  g.kb_per_split = (K / kBK + splits - 1) / splits;
  g.splits = (K / kBK + g.kb_per_split - 1) / g.kb_per_split;
  if (need(g.splits) > L.fused_bytes) throw std::invalid_argument("GEMM+allreduce: partials exceed the fused slot");
  g.fused = 1;
  if (g.m_tiles * g.n_tiles * g.splits > kMaxBlocks) throw std::invalid_argument("GEMM+allreduce: too many tiles");
  for (int r = 0; r < c.world_size(); ++r) g.wsp[r] = c.wsp(r);
  g.rank = c.rank();
  g.ws = c.world_size();
  g.slot_off = L.fused_off;
  g.slot_bytes = L.fused_bytes;
  g.err = c.err_dev();
  g.err_host = c.err_host();
  g.timeout_ns = c.config().timeout_ns;
  launch(wt, x, g, bn, s);
  c.count_launch();
  slots_rmsnorm(c, s, residual, weight, out, T, N, eps, g.splits);
  return g.splits;
}

}  // namespace nab

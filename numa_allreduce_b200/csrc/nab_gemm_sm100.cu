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
// Split-K: the `splits` CTAs of one output tile (at most 16) form a thread-
// block cluster. Each leaves its fp32 accumulator tile in its own shared
// memory; after a cluster barrier every CTA adds one slice of the tile over
// all splits in split order (distributed shared memory loads), so the
// reduction needs no global workspace and no second kernel.
//
// Programmatic dependent launch: the producer fills the ring with weight
// tiles before griddepcontrol.wait, so the weight stream of a decode-step
// GEMM starts while the kernel before it is still running.
//
// Fused with the allreduce (no counterpart in the reference, which has no
// fused ops): each slice is stored straight into this rank's slot on every
// rank over NVLink (its own included); once the whole tile is stored the
// tile's flag is raised on every rank. A second kernel waits for the flags of
// each row's tiles and adds the ranks' rows in rank order with the residual,
// then applies RMSNorm. The GEMM itself never waits for a peer.
//
// Every mbarrier and flag wait is bounded; on expiry the CTA stops issuing,
// waits (bounded) for its TMA loads in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "nab_comm.h"
#include "nab_driver.h"
#include "nab_fused.h"
#include "nab_gemm.h"
#include "nab_kerr.h"
#include "nab_proto.cuh"
#include "nab_sm100.cuh"

namespace nab {

namespace {

constexpr int kGemmThreads = 192;
constexpr int kBM = 128;
constexpr int kBK = 64;  // 128 bytes of bf16: one swizzle atom row
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMaxSplits = 16;  // CTAs per output tile = cluster size (16 needs the non-portable opt-in)

struct GemmArgs {
  int M;          // output features (rows of Wt), multiple of 128
  int K;          // multiple of 64
  int T;          // tokens
  int m_tiles;
  int n_tiles;
  int splits;     // CTAs per output tile = cluster size (1..16)
  int kb_per_split;
  int fused;
  int a_packed;   // Wt stored as contiguous 128 x 64 tiles (pack_weight layout)
  int swiglu;     // each 128-row tile is 64 gate rows then the 64 matching up
                  // rows; out[T, M/2] = silu(gate) * up
  __nv_bfloat16* out;  // [T, M] bf16 (not fused)
  // fused allreduce epilogue
  char* wsp[kMaxRanks];
  int rank;
  int ws;
  int64_t slot_off;    // fused one-shot slots: [2 parities][ws][slot_bytes]
  int64_t slot_bytes;
  int rs;              // reduce-scatter epilogue: token row t goes only to rank t % ws
  ErrorState* err;
  uint32_t* err_host;
  uint64_t timeout_ns;
};

// Small token tiles (decode) are bound by streaming the weight: 2 CTAs per SM
// with a shorter ring keep more bytes in flight per SM than one CTA with a
// long ring. Larger tiles use one CTA per SM and a deeper ring. The ring must
// also hold the fp32 accumulator tile [BN][128] for the split-K exchange.
template <int BN>
struct GemmCfg {
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN == 16 ? 6 : (BN == 32 ? 5 : (BN == 64 ? 8 : (BN == 128 ? 6 : 4)));
  static constexpr int kCtasPerSm = BN <= 32 ? 2 : 1;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024;  // + alignment slack
  static_assert(kStages * kStageBytes >= BN * kBM * 4, "accumulator tile must fit the ring");
};

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, GemmCfg<BN>::kCtasPerSm)
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
  __shared__ uint32_t s_epoch;
  volatile int* abort_flag = &s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the splits of one output tile are consecutive CTAs: one cluster
  const int split = blockIdx.x % g.splits;
  const int tile = blockIdx.x / g.splits;
  const int m_tile = tile % g.m_tiles;
  const int n_tile = tile / g.m_tiles;
  const int m0 = m_tile * kBM;
  const int t0 = n_tile * BN;
  const int kb0 = split * g.kb_per_split;
  const int kb1 = min(g.K / kBK, kb0 + g.kb_per_split);
  const int nkb = max(0, kb1 - kb0);
  const int rows = min(BN, g.T - t0);  // valid tokens of this tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    sm100::mbar_init(&accum_bar, 1);
    sm100::fence_barrier_init();
    s_abort = 0;
    s_epoch = 0;
    sm100::prefetch_tensormap(&tmA);
    sm100::prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    sm100::tmem_alloc(&s_tmem, Cfg::kTmemCols);
    sm100::tmem_relinquish();
  }
  // a programmatically dependent launch after this one may start scheduling
  // (it still waits for this grid to complete before it reads our output)
  if (threadIdx.x == 0) sm100::griddep_launch_dependents();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = s_tmem;

  // A wait that ran out: the fused kernel records on its communicator (and
  // stops this rank's other waits), the plain one on the device's kernel
  // error record.
  auto fail = [&](uint32_t stage) {
    if (!*abort_flag) {
      if (g.fused) {
        WaitCtx w = make_wait(g.err, g.err_host, g.timeout_ns, g.wsp, g.rank, 0);
        record_failure(w, kErrTimeout, static_cast<uint32_t>(g.rank), stage, 0);
      } else {
        record_local_failure(g.err, g.err_host, kErrTimeout, stage, 0);
      }
    }
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      // weight tile (m_tile, kb): row-major Wt, or the packed layout in which
      // each 128 x 64 tile is 16 KB of contiguous memory (one DRAM stream)
      auto a_x = [&](int kb) { return g.a_packed ? 0 : kb * kBK; };
      auto a_y = [&](int kb) { return g.a_packed ? (m_tile * (g.K / kBK) + kb) * kBM : m0; };
      // The weight does not depend on the previous kernel in the stream:
      // fill the ring with weight tiles first, and only then wait (with a
      // programmatic dependent launch) for the activations to be ready.
      const int pre = min(S, nkb);
      for (int i = 0; i < pre; ++i) {
        uint8_t* sa = smem + i * Cfg::kStageBytes;
        sm100::mbar_arrive_expect_tx(&full_bar[i], Cfg::kStageBytes);
        sm100::tma_load_2d(sa, &tmA, a_x(kb0 + i), a_y(kb0 + i), &full_bar[i]);
      }
      sm100::griddep_wait();
      for (int i = 0; i < pre; ++i)
        sm100::tma_load_2d(smem + i * Cfg::kStageBytes + kABytes, &tmB, (kb0 + i) * kBK, t0, &full_bar[i]);
      int issued = pre;
      for (int i = pre; i < nkb; ++i) {
        const int s = i % S;
        if (!sm100::mbar_wait(&empty_bar[s], ((i / S) - 1) & 1, g.timeout_ns, abort_flag)) {
          fail(g.fused ? kStageGemmAR : kStageGemm);
          break;
        }
        if (*abort_flag) break;
        uint8_t* sa = smem + s * Cfg::kStageBytes;
        sm100::mbar_arrive_expect_tx(&full_bar[s], Cfg::kStageBytes);
        sm100::tma_load_2d(sa, &tmA, a_x(kb0 + i), a_y(kb0 + i), &full_bar[s]);
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
          fail(g.fused ? kStageGemmAR : kStageGemm);
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
    // ------------------------------------- epilogue, part 1: TMEM -> smem
    // The accumulator goes to this CTA's (now idle) ring as fp32
    // [token][feature]; a split with no k-blocks contributes zeros.
    const int q = warp & 3;        // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;  // feature within the tile
    if (nkb > 0 && !sm100::mbar_wait(&accum_bar, 0, g.timeout_ns, abort_flag)) fail(g.fused ? kStageGemmAR : kStageGemm);
    sm100::tc_fence_after();
    float* acc = reinterpret_cast<float*>(smem);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      if (c0 >= rows) break;
      uint32_t r[16];
      if (nkb > 0) {
        sm100::tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
        sm100::tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[(c0 + j) * kBM + row] = __uint_as_float(r[j]);
    }
    if (g.fused && threadIdx.x == 64) {
      // The epoch of the previous call is final once the kernels before
      // this launch have completed.
      sm100::griddep_wait();
      s_epoch = ld_volatile_u32(&pad_at(g.wsp, g.rank)->epoch) + 1u;
    }
  }
  // All splits' accumulators are in their CTAs' shared memory.
  sm100::tc_fence_before();
  if (g.splits > 1) sm100::cluster_sync(); else __syncthreads();

  // ------------------------------ epilogue, part 2: split reduce + store
  // The tile's output is [rows][128] features (64 with SwiGLU) = chunks of
  // 8; the cluster's CTAs take contiguous ranges of chunks, add the splits'
  // fp32 values in split order (every CTA of the cluster holds one split)
  // and write bf16.
  const bool ok = !*abort_flag;
  if (warp >= 2 && ok) {
    const int et = threadIdx.x - 64;
    const int out_cols = g.swiglu ? kBM / 2 : kBM;
    const int ldo = g.swiglu ? g.M / 2 : g.M;  // output row stride
    const int cpr = out_cols / 8;               // chunks per token row
    const int nchunk = rows * cpr;
    const int per = (nchunk + g.splits - 1) / g.splits;
    const int c_beg = split * per, c_end = min(nchunk, c_beg + per);
    const uint32_t acc_addr = sm100::smem_u32(smem);
    const int parity = s_epoch & 1;
    // 8 consecutive fp32 accumulator values at byte offset `off`, summed over
    // the splits in split order
    auto gather8 = [&](uint32_t off, float (&v)[8]) {
      if (g.splits == 1) {
        const float4 lo = *reinterpret_cast<const float4*>(smem + off);
        const float4 hi = *reinterpret_cast<const float4*>(smem + off + 16);
        v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
        v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
        return;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
      for (int sp = 0; sp < g.splits; ++sp) {
        const uint32_t ra = sm100::dsmem_addr(acc_addr + off, static_cast<uint32_t>(sp));
        const float4 lo = sm100::ld_dsmem_f4(ra), hi = sm100::ld_dsmem_f4(ra + 16);
        v[0] += lo.x; v[1] += lo.y; v[2] += lo.z; v[3] += lo.w;
        v[4] += hi.x; v[5] += hi.y; v[6] += hi.z; v[7] += hi.w;
      }
    };
    for (int c = c_beg + et; c < c_end; c += 128) {
      const int t = c / cpr, f = (c % cpr) * 8;
      float v[8];
      gather8(static_cast<uint32_t>((t * kBM + f) * 4), v);
      if (g.swiglu) {
        float u[8];
        gather8(static_cast<uint32_t>((t * kBM + kBM / 2 + f) * 4), u);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = v[j] / (1.f + __expf(-v[j])) * u[j];
      }
      uint4 packed;
      __nv_bfloat162 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      packed.x = *reinterpret_cast<uint32_t*>(&h[0]);
      packed.y = *reinterpret_cast<uint32_t*>(&h[1]);
      packed.z = *reinterpret_cast<uint32_t*>(&h[2]);
      packed.w = *reinterpret_cast<uint32_t*>(&h[3]);
      const int64_t eoff = static_cast<int64_t>(t0 + t) * ldo + m_tile * out_cols + f;  // element offset
      if (!g.fused) {
        *reinterpret_cast<uint4*>(g.out + eoff) = packed;
      } else if (g.rs) {
        // reduce-scatter by stores: only the row's owner gets it
        const int dst = (t0 + t) % g.ws;
        char* slot = g.wsp[dst] + g.slot_off + (static_cast<int64_t>(parity) * g.ws + g.rank) * g.slot_bytes;
        *reinterpret_cast<uint4*>(slot + eoff * 2) = packed;
      } else {
        // into this rank's slot on every rank (its own included), staggered
        for (int k = 0; k < g.ws; ++k) {
          const int dst = (g.rank + k) % g.ws;
          char* slot = g.wsp[dst] + g.slot_off + (static_cast<int64_t>(parity) * g.ws + g.rank) * g.slot_bytes;
          *reinterpret_cast<uint4*>(slot + eoff * 2) = packed;
        }
      }
    }
  }
  // No CTA leaves while a peer of its cluster may still read its shared
  // memory; with the allreduce, every slice of the tile is stored.
  if (g.splits > 1) sm100::cluster_sync(); else __syncthreads();
  if (g.fused && split == 0 && threadIdx.x < g.ws && !*abort_flag) {
    // the tile is in every rank: raise its flag there (the norm kernel waits)
    const int dst = (g.rank + threadIdx.x) % g.ws;
    st_release_sys(&pad_at(g.wsp, dst)->gemm_flags[n_tile * g.m_tiles + m_tile][g.rank], make_seq(s_epoch, 0));
  }
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (g.fused) end_call(g.wsp, g.rank, s_epoch);
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

// Launch with the split CTAs of a tile as one thread-block cluster and, when
// `pdl`, as a programmatic dependent launch (the weight prefetch overlaps the
// tail of the previous kernel in the stream).
template <int BN>
void launch_bn(const CUtensorMap& a, const CUtensorMap& b, const GemmArgs& g, int grid, cudaStream_t s, bool pdl) {
  using Cfg = GemmCfg<BN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    NAB_CUDA_CHECK(cudaFuncSetAttribute(k_gemm_bf16<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem));
    NAB_CUDA_CHECK(cudaFuncSetAttribute(k_gemm_bf16<BN>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    attr_set[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  attrs[n].id = cudaLaunchAttributeClusterDimension;
  attrs[n].val.clusterDim.x = g.splits;
  attrs[n].val.clusterDim.y = 1;
  attrs[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_bf16<BN>, a, b, g);
  if (e != cudaSuccess) throw std::runtime_error(std::string("GEMM launch failed: ") + cudaGetErrorString(e));
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("NAB_GEMM_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

void launch(const void* wt, const void* x, const GemmArgs& g, int bn, cudaStream_t s) {
  const CUtensorMap a = g.a_packed ? make_map(wt, static_cast<int64_t>(g.M) * (g.K / kBK), kBK, kBM)
                                   : make_map(wt, g.M, g.K, kBM);
  const CUtensorMap b = make_map(x, g.T, g.K, bn);
  const int grid = g.m_tiles * g.n_tiles * g.splits;
  const bool pdl = pdl_enabled();
  switch (bn) {
    case 16: launch_bn<16>(a, b, g, grid, s, pdl); break;
    case 32: launch_bn<32>(a, b, g, grid, s, pdl); break;
    case 64: launch_bn<64>(a, b, g, grid, s, pdl); break;
    case 128: launch_bn<128>(a, b, g, grid, s, pdl); break;
    default: launch_bn<256>(a, b, g, grid, s, pdl); break;
  }
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// Clusters of `cs` CTAs of the BN-wide kernel that fit on the device at once
// (cudaOccupancyMaxActiveClusters: accounts for shared memory, CTAs per SM
// and the placement of a cluster inside one GPC). 0 if it cannot launch.
template <int BN>
int active_clusters_bn(int cs) {
  using Cfg = GemmCfg<BN>;
  NAB_CUDA_CHECK(cudaFuncSetAttribute(k_gemm_bf16<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem));
  NAB_CUDA_CHECK(cudaFuncSetAttribute(k_gemm_bf16<BN>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(cs * 64);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = cs;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k_gemm_bf16<BN>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int active_clusters(int bn, int cs) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;  // (device, bn, cs) -> clusters
  int dev = 0;
  cudaGetDevice(&dev);
  const int key = (dev << 16) | (bn << 5) | cs;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  switch (bn) {
    case 16: n = active_clusters_bn<16>(cs); break;
    case 32: n = active_clusters_bn<32>(cs); break;
    case 64: n = active_clusters_bn<64>(cs); break;
    case 128: n = active_clusters_bn<128>(cs); break;
    default: n = active_clusters_bn<256>(cs); break;
  }
  cache[key] = n;
  return n;
}

// Split count actually launched: every split gets at least one k-block.
void set_splits(GemmArgs& g, int splits, int bn) {
  const int kb = g.K / kBK;
  splits = std::max(1, std::min({splits, kMaxSplits, kb}));
  while (splits > 1 && active_clusters(bn, splits) == 0) --splits;
  g.kb_per_split = (kb + splits - 1) / splits;
  g.splits = (kb + g.kb_per_split - 1) / g.kb_per_split;
}

void check_shape(int T, int N, int K) {
  if (T < 1 || N < kBM || N % kBM != 0 || K < kBK || K % kBK != 0)
    throw std::invalid_argument("GEMM needs T >= 1, N a multiple of 128 and K a multiple of 64");
}

}  // namespace

int gemm_active_clusters(int bn, int cs) { return active_clusters(bn, cs); }

int gemm_ar_mode_for(int T, int ws) {
  // One-shot: every rank's whole output crosses to every peer ((ws - 1) T H
  // elements per direction) but needs no second exchange; reduce-scatter +
  // gather moves 2 (ws - 1) / ws T H and adds one flag round trip. At two
  // ranks both move the same bytes; measured at 4 and 8 ranks (Llama-3-8B
  // down projection) the one-shot led up to 128 tokens, so the
  // reduce-scatter is taken only for larger outputs.
  if (ws <= 2) return kGemmArOneshot;
  return T >= 256 ? kGemmArReduceScatter : kGemmArOneshot;
}

namespace {

// Split rule "waves": a time model in k-blocks, waves of co-resident
// clusters x (k-blocks per split + a fixed cost per CTA for its prologue and
// epilogue); ties go to fewer splits.
int splits_waves(int bn, int tiles, int kb) {
  const int fixed = bn <= 32 ? 3 : 2;
  int best = 1;
  int64_t best_cost = INT64_MAX;
  for (int sp = 1; sp <= kMaxSplits && sp <= kb; ++sp) {
    const int per = (kb + sp - 1) / sp;
    if ((kb + per - 1) / per != sp) continue;  // would leave a split without work
    const int clusters = active_clusters(bn, sp);
    if (clusters == 0) continue;
    const int64_t waves = (tiles + clusters - 1) / clusters;
    const int64_t cost = waves * (per + fixed);
    if (cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

// Split rule "fill": fill every CTA slot of the device once, the largest
// split count with tiles x splits <= CTAs per SM x SMs and at least 8
// k-blocks per split, clusters of at most 8 CTAs when one CTA fills an SM.
// Best or within a few percent of the best for a GEMM that has the device to
// itself (bench/gemm.py --split-sweep, Llama-3-70B TP-8 projections), but
// slower than both other rules inside a decode step.
int splits_fill(int bn, int tiles, int kb, int sms) {
  const int per_sm = bn <= 32 ? 2 : 1;
  const int cap = std::min({bn <= 32 ? kMaxSplits : 8, std::max(1, (per_sm * sms) / tiles), std::max(1, kb / 8)});
  for (int sp = cap; sp > 1; --sp) {
    const int per = (kb + sp - 1) / sp;
    if ((kb + per - 1) / per != sp) continue;
    if (active_clusters(bn, sp) == 0) continue;
    return sp;
  }
  return 1;
}

// Split rule "pow2" (the default): the largest power of two with tiles x
// splits <= CTA
// slots of the device (2 per SM when the tile is at most 32 tokens wide, else
// 1), at least 2 k-blocks per split, clusters of at most 16 (8 when one CTA
// fills an SM). A cluster of 5-7 CTAs at one CTA per SM packs badly into
// the GPCs (Llama-3-8B gate|up at 64 tokens: 12.0 us at 4 splits, 20.3 us at
// 5). Within 8 % of the best count on every Llama-3-8B / 70B TP-8 projection
// at 1-128 tokens measured alone on the device, and the fastest of the three
// rules inside the Llama-3-70B TP-8 decode step (one GPU's shard, CUDA graph:
// 5.19 / 6.35 ms per token at batch 1 / 32 against 5.71 / 6.53 for "waves"
// and 6.07 / 6.76 for "fill").
int splits_pow2(int bn, int tiles, int kb, int sms) {
  const int per_sm = bn <= 32 ? 2 : 1;
  const int cap = std::min({bn <= 32 ? kMaxSplits : 8, std::max(1, (per_sm * sms) / tiles), std::max(1, kb / 2)});
  int sp = 1;
  while (sp * 2 <= cap) sp *= 2;
  for (; sp > 1; sp /= 2) {
    const int per = (kb + sp - 1) / sp;
    if ((kb + per - 1) / per != sp) continue;
    if (active_clusters(bn, sp) == 0) continue;
    return sp;
  }
  return 1;
}

enum SplitRule { kSplitWaves, kSplitFill, kSplitPow2 };

SplitRule split_rule() {
  static const SplitRule rule = [] {
    const char* v = std::getenv("NAB_GEMM_SPLIT_RULE");
    if (v != nullptr && std::strcmp(v, "fill") == 0) return kSplitFill;
    if (v != nullptr && std::strcmp(v, "waves") == 0) return kSplitWaves;
    return kSplitPow2;
  }();
  return rule;
}

}  // namespace

int gemm_splits_for(int T, int N, int K, int sms) {
  if (sms <= 0) sms = sm_count();
  const int bn = pick_bn(T);
  const int tiles = (N / kBM) * ((T + bn - 1) / bn);
  const int kb = K / kBK;
  switch (split_rule()) {
    case kSplitFill: return splits_fill(bn, tiles, kb, sms);
    case kSplitWaves: return splits_waves(bn, tiles, kb);
    default: return splits_pow2(bn, tiles, kb, sms);  // kSplitPow2
  }
}

void gemm_bf16(cudaStream_t s, const void* wt, const void* x, void* y, int T, int N, int K, int splits,
               bool packed, bool swiglu) {
  check_shape(T, N, K);
  GemmArgs g{};
  g.a_packed = packed ? 1 : 0;
  g.swiglu = swiglu ? 1 : 0;
  const int bn = pick_bn(T);
  g.M = N;
  g.K = K;
  g.T = T;
  g.m_tiles = N / kBM;
  g.n_tiles = (T + bn - 1) / bn;
  set_splits(g, splits > 0 ? splits : gemm_splits_for(T, N, K, sm_count()), bn);
  g.out = static_cast<__nv_bfloat16*>(y);
  const KernelErrorRecord rec = kernel_error_record();
  g.err = rec.dev;
  g.err_host = rec.host;
  g.timeout_ns = kernel_timeout_ns();
  launch(wt, x, g, bn, s);
}

int gemm_allreduce_rmsnorm(Communicator& c, cudaStream_t s, const void* wt, const void* x, void* residual,
                           const void* weight, void* out, int T, int N, int K, float eps, int splits, bool packed,
                           int mode) {
  check_shape(T, N, K);
  const Layout& L = c.layout();
  if (c.world_size() == 1) throw std::invalid_argument("GEMM+allreduce needs a world size of at least 2");
  if (static_cast<int64_t>(T) * N * 2 > L.fused_bytes)
    throw std::invalid_argument("GEMM+allreduce: the output exceeds the fused slot");
  const int bn = pick_bn(T);
  GemmArgs g{};
  g.M = N;
  g.K = K;
  g.T = T;
  g.m_tiles = N / kBM;
  g.n_tiles = (T + bn - 1) / bn;
  if (g.m_tiles * g.n_tiles > kGemmMaxTiles) throw std::invalid_argument("GEMM+allreduce: too many output tiles");
  set_splits(g, splits > 0 ? splits : gemm_splits_for(T, N, K, sm_count()), bn);
  g.fused = 1;
  g.a_packed = packed ? 1 : 0;
  for (int r = 0; r < c.world_size(); ++r) g.wsp[r] = c.wsp(r);
  g.rank = c.rank();
  g.ws = c.world_size();
  g.slot_off = L.fused_off;
  g.slot_bytes = L.fused_bytes;
  g.err = c.err_dev();
  g.err_host = c.err_host();
  g.timeout_ns = c.config().timeout_ns;
  if (mode == kGemmArAuto) mode = gemm_ar_mode_for(T, c.world_size());
  g.rs = mode == kGemmArReduceScatter ? 1 : 0;
  launch(wt, x, g, bn, s);
  c.count_launch();
  if (g.rs)
    slots_rs_rmsnorm(c, s, residual, weight, out, T, N, eps, bn);
  else
    slots_rmsnorm(c, s, residual, weight, out, T, N, eps, bn);
  return g.splits;
}

}  // namespace nab

// Device-side building blocks: 16-byte packs with fp32 accumulation, flag
// loads/stores with sys-scope release/acquire, bounded waits that record an
// error instead of hanging, and the NVLink-SHARP (multimem) primitives.
//
// Capability parity: the reference's packed vector math (array_t/packed_t,
// upcast/downcast, packed_reduce; src/numa_all_reduce.cu:75-146,215-223) and
// its volatile flag barrier (src/numa_all_reduce.cu:149-212). Differences by
// design: flags use st.release.sys / ld.acquire.sys instead of volatile
// accesses without fences, every wait is bounded by %globaltimer, and values
// are 64-bit sequence numbers so a stale flag can never look current.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "nab_common.h"

#define NAB_DINLINE __device__ __forceinline__

// Debug builds (-DNAB_DEBUG_BOUNDS=1) check launch parameters, slot capacity,
// ranks and pack indices on the device; a violation is recorded (code
// kErrBadLaunch, stage kStageBounds) and the guarded access is skipped. No
// trap, no assert. Release builds compile the checks away.
#include "nab_device_flags.h"

namespace nab {

// ---------------------------------------------------------------- packs ----
template <typename T>
struct VecT;
template <>
struct VecT<float> {
  static constexpr int kN = 4;
};
template <>
struct VecT<__half> {
  static constexpr int kN = 8;
};
template <>
struct VecT<__nv_bfloat16> {
  static constexpr int kN = 8;
};

template <typename T>
struct Acc {
  float v[VecT<T>::kN];
};

NAB_DINLINE void acc_set(Acc<float>& a, uint4 x) {
  a.v[0] = __uint_as_float(x.x);
  a.v[1] = __uint_as_float(x.y);
  a.v[2] = __uint_as_float(x.z);
  a.v[3] = __uint_as_float(x.w);
}
NAB_DINLINE void acc_add(Acc<float>& a, uint4 x) {
  a.v[0] += __uint_as_float(x.x);
  a.v[1] += __uint_as_float(x.y);
  a.v[2] += __uint_as_float(x.z);
  a.v[3] += __uint_as_float(x.w);
}
NAB_DINLINE uint4 acc_pack(const Acc<float>& a) {
  return make_uint4(__float_as_uint(a.v[0]), __float_as_uint(a.v[1]),
                    __float_as_uint(a.v[2]), __float_as_uint(a.v[3]));
}

// bf16 -> f32 is exact: the bf16 bits are the high half of the f32 bits.
NAB_DINLINE void acc_set(Acc<__nv_bfloat16>& a, uint4 x) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    a.v[2 * k] = __uint_as_float(w[k] << 16);
    a.v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}
NAB_DINLINE void acc_add(Acc<__nv_bfloat16>& a, uint4 x) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    a.v[2 * k] += __uint_as_float(w[k] << 16);
    a.v[2 * k + 1] += __uint_as_float(w[k] & 0xffff0000u);
  }
}
NAB_DINLINE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
NAB_DINLINE uint4 acc_pack(const Acc<__nv_bfloat16>& a) {
  return make_uint4(pack_bf16x2(a.v[0], a.v[1]), pack_bf16x2(a.v[2], a.v[3]),
                    pack_bf16x2(a.v[4], a.v[5]), pack_bf16x2(a.v[6], a.v[7]));
}

NAB_DINLINE void acc_set(Acc<__half>& a, uint4 x) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
    float2 f = __half22float2(h);
    a.v[2 * k] = f.x;
    a.v[2 * k + 1] = f.y;
  }
}
NAB_DINLINE void acc_add(Acc<__half>& a, uint4 x) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
    float2 f = __half22float2(h);
    a.v[2 * k] += f.x;
    a.v[2 * k + 1] += f.y;
  }
}
NAB_DINLINE uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
NAB_DINLINE uint4 acc_pack(const Acc<__half>& a) {
  return make_uint4(pack_f16x2(a.v[0], a.v[1]), pack_f16x2(a.v[2], a.v[3]),
                    pack_f16x2(a.v[4], a.v[5]), pack_f16x2(a.v[6], a.v[7]));
}

// fp32 image of an accumulator, as kN / 4 packs (1 for fp32, 2 for 16-bit types).
template <typename T>
struct AccWords {
  static constexpr int kW = VecT<T>::kN / 4;
};

template <typename T>
NAB_DINLINE void acc_store_f32(uint4* p, const Acc<T>& a) {
#pragma unroll
  for (int w = 0; w < AccWords<T>::kW; ++w)
    p[w] = make_uint4(__float_as_uint(a.v[4 * w]), __float_as_uint(a.v[4 * w + 1]),
                      __float_as_uint(a.v[4 * w + 2]), __float_as_uint(a.v[4 * w + 3]));
}

// a = (first ? 0 : a) + the fp32 image at p, read through L2 only.
template <typename T>
NAB_DINLINE void acc_accum_f32(Acc<T>& a, const uint4* p, bool first) {
#pragma unroll
  for (int w = 0; w < AccWords<T>::kW; ++w) {
    const uint4 x = __ldcg(p + w);
    const float f[4] = {__uint_as_float(x.x), __uint_as_float(x.y), __uint_as_float(x.z), __uint_as_float(x.w)};
#pragma unroll
    for (int e = 0; e < 4; ++e) a.v[4 * w + e] = first ? f[e] : a.v[4 * w + e] + f[e];
  }
}

// --------------------------------------------------------- memory access ----
// Data loads of buffers that another GPU wrote during this kernel go through
// L2 only (.cg) so a line cached in L1 by an earlier round is never reused.
NAB_DINLINE uint4 ld_cg(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
NAB_DINLINE uint4 ld_plain(const void* p) { return *reinterpret_cast<const uint4*>(p); }
NAB_DINLINE void st_plain(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

NAB_DINLINE void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
NAB_DINLINE uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
NAB_DINLINE uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
NAB_DINLINE uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
NAB_DINLINE void st_volatile_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Named barrier over `n` threads that also ORs a predicate over them: every
// participating thread gets the same answer, so a group can leave a loop
// together even when a flag it reads may change while its threads arrive.
NAB_DINLINE bool named_barrier_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// Programmatic dependent launch: lets a kernel launched after this one with
// programmatic stream serialization begin scheduling now (it waits for this
// grid's completion before it reads anything this grid writes).
NAB_DINLINE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits for the grids this launch programmatically depends on to complete
// (no-op without such a dependency).
NAB_DINLINE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

NAB_DINLINE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------- NVLink SHARP ops ----
// multimem.* take a multicast virtual address: loads are reduced inside the
// NVSwitch across every GPU bound to the object, stores are replicated to all.
template <typename T>
NAB_DINLINE uint4 mm_ld_reduce(const void* mc);
template <>
NAB_DINLINE uint4 mm_ld_reduce<__nv_bfloat16>(const void* mc) {
  uint4 r;
  asm volatile(
      "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(mc)
      : "memory");
  return r;
}
template <>
NAB_DINLINE uint4 mm_ld_reduce<__half>(const void* mc) {
  uint4 r;
  asm volatile(
      "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(mc)
      : "memory");
  return r;
}
template <>
NAB_DINLINE uint4 mm_ld_reduce<float>(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
template <typename T>
NAB_DINLINE void mm_st(void* mc, uint4 v);
template <>
NAB_DINLINE void mm_st<__nv_bfloat16>(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
template <>
NAB_DINLINE void mm_st<__half>(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
template <>
NAB_DINLINE void mm_st<float>(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
// Orders this thread's accesses made through one virtual alias of a physical
// location (e.g. the unicast address of the NVLS workspace) with its accesses
// through another alias of it (the multicast address).
NAB_DINLINE void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Increments the counter at the same offset on every GPU of the multicast
// object. Release: the CTA's earlier writes (ordered by bar.sync) are visible
// to any GPU that acquires the incremented value.
NAB_DINLINE void mm_red_add_release(uint32_t* mc, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

// ----------------------------------------------------------- bounded waits --
struct WaitCtx {
  ErrorState* err;      // device memory, shared by the CTAs of this launch
  uint32_t* err_host;   // host-mapped copy of the error code (may be null)
  uint32_t* abort;      // this rank's abort word (in its signal pad)
  uint64_t timeout_ns;
  uint32_t rank;
  uint32_t epoch;
};

// Records the first failure with its details; later ones only bump the count.
NAB_DINLINE void record_failure(const WaitCtx& w, uint32_t code, uint32_t peer, uint32_t stage,
                                uint32_t observed) {
  if (atomicCAS(&w.err->code, 0u, code) == 0u) {
    w.err->rank = w.rank;
    w.err->peer = peer;
    w.err->stage = stage;
    w.err->block = blockIdx.x;
    w.err->epoch = w.epoch;
    w.err->observed = observed;
    __threadfence_system();
    if (w.err_host) st_volatile_u32(w.err_host, code);
  }
  atomicAdd(&w.err->count, 1u);
  st_volatile_u32(w.abort, 1u);
}

// Records a failure of a kernel that has no communicator (no peers to stop):
// the first one fills the record, later ones only bump the count.
NAB_DINLINE void record_local_failure(ErrorState* err, uint32_t* err_host, uint32_t code, uint32_t stage,
                                      uint32_t observed) {
  if (err == nullptr) return;
  if (atomicCAS(&err->code, 0u, code) == 0u) {
    err->rank = 0xffffffffu;
    err->peer = 0xffffffffu;
    err->stage = stage;
    err->block = blockIdx.x + gridDim.x * blockIdx.y;
    err->epoch = 0;
    err->observed = observed;
    __threadfence_system();
    if (err_host) st_volatile_u32(err_host, code);
  }
  atomicAdd(&err->count, 1u);
}

// Debug builds: true if `cond` holds; otherwise records the violation (with
// `observed`, e.g. the offending index) and returns false. Always true in
// release builds.
NAB_DINLINE bool dbg_ok(bool cond, ErrorState* err, uint32_t* err_host, uint32_t observed) {
  if (!NAB_DEBUG_BOUNDS || cond) return true;
  record_local_failure(err, err_host, kErrBadLaunch, kStageBounds, observed);
  return false;
}

// Spins until *addr >= target (wrap-safe). Returns false, after recording the
// failure, once the wait has run longer than the timeout or another CTA of
// this rank has already given up.
NAB_DINLINE bool wait_geq(const uint64_t* addr, uint64_t target, const WaitCtx& w,
                          uint32_t peer, uint32_t stage) {
  uint64_t v = ld_acquire_sys(addr);
  if (static_cast<int64_t>(v - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    v = ld_acquire_sys(addr);
    if (static_cast<int64_t>(v - target) >= 0) return true;
    if ((it & 255u) == 0u) {
      if (ld_volatile_u32(w.abort) != 0u) return false;
      if (globaltimer_ns() - t0 > w.timeout_ns) {
        record_failure(w, kErrTimeout, peer, stage, static_cast<uint32_t>(v));
        return false;
      }
    }
  }
}

// Same for a 32-bit counter (NVLS arrival counters).
NAB_DINLINE bool wait_geq_u32(const uint32_t* addr, uint32_t target, const WaitCtx& w,
                              uint32_t stage) {
  uint32_t v = ld_acquire_sys_u32(addr);
  if (static_cast<int32_t>(v - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    v = ld_acquire_sys_u32(addr);
    if (static_cast<int32_t>(v - target) >= 0) return true;
    if ((it & 255u) == 0u) {
      if (ld_volatile_u32(w.abort) != 0u) return false;
      if (globaltimer_ns() - t0 > w.timeout_ns) {
        record_failure(w, kErrTimeout, 0xffffffffu, stage, v);
        return false;
      }
    }
  }
}

// min(cap, avail) clamped at 0: the valid length of a ragged last piece.
NAB_DINLINE int64_t span_len(int64_t cap, int64_t avail) {
  const int64_t v = cap < avail ? cap : avail;
  return v > 0 ? v : 0;
}

template <typename T>
NAB_DINLINE T ceil_div(T a, T b) {
  return (a + b - 1) / b;
}

}  // namespace nab

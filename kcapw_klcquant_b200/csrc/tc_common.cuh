// sm_100a building blocks shared by the tensor-core kernels: mbarriers with
// bounded waits, TMA / bulk copies, tcgen05 (MMA, commit, TMEM loads, shared
// memory -> TMEM copies), shared-memory matrix descriptors and tensor-map
// encoding through the driver entry point.
//
// Every wait is bounded: after kWaitCycles SM cycles the waiting role records
// KLC_ERR_DEVICE_TIMEOUT in the workspace status word and raises a CTA-wide
// abort flag; drains after an abort are bounded by kWaitNs of %globaltimer.
#pragma once

#include <cuda.h>

#include "klc_common.cuh"

namespace klc {
namespace tc {

constexpr uint64_t kWaitNs = 2000000000ull;      // drain bound: 2 s of %globaltimer
constexpr long long kWaitCycles = 4000000000ll;  // wait bound: 4e9 SM cycles (2 s at 2 GHz)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

struct Ctl {
  volatile int* abort;
  DeviceStatus* status;
};

// Bounded wait for the completion of phase `parity` of a barrier.  Returns
// false when the CTA is aborting (this wait timed out or another did).
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const Ctl& c, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  // the SM cycle counter is cheap to read; the bound is checked every 64 polls
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*c.abort) return false;
      if (clock64() - t0 > kWaitCycles) {
        *c.abort = 1;
        record_fault(c.status, KLC_ERR_DEVICE_TIMEOUT, site, 0);
        return false;
      }
    }
  }
}

// Bounded wait with an explicit cycle limit (the wait self-test uses a short one).
__device__ __forceinline__ bool wait_bar_limit(uint32_t bar, uint32_t parity, const Ctl& c, int site, long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*c.abort) return false;
    if (clock64() - t0 > limit) {
      *c.abort = 1;
      record_fault(c.status, KLC_ERR_DEVICE_TIMEOUT, site, 0);
      return false;
    }
  }
  return true;
}

// Bounded wait for roles that wait long and are not on the critical path:
// sleeping between polls leaves issue slots to the warps that share the
// scheduler (the MMA issuer above all).
__device__ __forceinline__ bool wait_bar_backoff(uint32_t bar, uint32_t parity, const Ctl& c, int site) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*c.abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *c.abort = 1;
      record_fault(c.status, KLC_ERR_DEVICE_TIMEOUT, site, 0);
      return false;
    }
    __nanosleep(256);
  }
  return true;
}

// Drain-time wait: bounded, ignores the abort flag.
static __device__ __noinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) return;
    __nanosleep(64);
  }
}

// After an abort: wait (bounded) for the latest load issued into each slot of
// a ring of `n` full-barriers (8 bytes apart) that received `issued` loads in
// slot order (load i went to slot i % n, completing phase (i / n) & 1).
static __device__ __noinline__ void drain_ring(uint32_t full0, int n, uint32_t issued) {
  for (int s = 0; s < n; ++s) {
    if (issued <= uint32_t(s)) break;
    const uint32_t last = issued - 1 - ((issued - 1 - uint32_t(s)) % uint32_t(n));
    drain_wait(full0 + 8u * s, (last / uint32_t(n)) & 1);
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// L2 prefetch of a tensor box (no shared memory, no completion to wait for)
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// L2 prefetch of a contiguous range (16-byte aligned, a multiple of 16 bytes)
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// contiguous global -> shared copy; both addresses 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// generic-proxy shared-memory writes -> visible to the async proxy (tcgen05 / TMA)
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 4 columns of 32 bits from registers into TMEM (lanes of the
// calling warp's quarter: taddr carries lane 32 * (warp % 4))
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint4 v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row groups
// 1024 bytes apart (SBO), leading offset unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

// Shared-memory descriptor of a 32-row x 16-byte block without swizzle (8-row
// groups 128 bytes apart): the source of a 32x128b shared -> TMEM copy.
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(128 >> 4) << 32) | (uint64_t(1) << 46);
}

// Host: tensor-map encoding (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the library does not link libcuda).
int make_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);

}  // namespace tc
}  // namespace klc

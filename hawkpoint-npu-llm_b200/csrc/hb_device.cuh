// hb_device.cuh -- sm_100a device primitives for the weight-streaming kernels.
//
// * mbarrier + cp.async.bulk (untiled bulk copy, no cluster multicast) move
//   weight chunks from HBM into a shared-memory ring;
// * every wait (mbarrier phase, grid-barrier counter, test stall flag) is
//   bounded by %globaltimer: when the limit passes, the waiting thread records
//   an error code in the control block, raises the abort flag, and returns
//   false, so the kernel winds down and the host sees HB_ERR_DEVICE_TIMEOUT;
// * BF16 / int8 unpacking helpers for the FP32-accumulating dot products.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace hb {

// Control block in global memory, one per engine / GEMV scratch.
struct Ctrl {
  unsigned int bar;        // grid-barrier arrival counter (reset by the last CTA)
  unsigned int done;       // CTAs that finished the launch
  int err;                 // first error code (0 = none)
  int err_where;           // which wait gave up
  int abort;               // raised with err; every wait polls it
  int stall_flag;          // never set: the test stall waits on it
  int pad[2];
};

enum : int {
  kErrNone = 0,
  kErrTimeout = 1,
  kErrBadToken = 2,  // a device-chained token id fell outside the vocabulary
  kErrBadPage = 3,   // a KV page-table entry fell outside the page pool
};

enum : int {
  kWhereFull = 1,
  kWhereEmpty = 2,
  kWhereGrid = 3,
  kWhereStall = 4,
  kWhereDrain = 5,
  kWhereToken = 6,
  kWhereKvPage = 7,
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_volatile_int(const int *p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

static __device__ __noinline__ void raise_error(Ctrl *ctrl, int code, int where) {
  if (atomicCAS(&ctrl->err, 0, code) == 0) {
    atomicExch(&ctrl->err_where, where);
  }
  atomicExch(&ctrl->abort, 1);
}

// The slow half of every bounded wait, kept out of line so that wait sites
// compile to a load and a compare: true when the wait must give up because
// another CTA raised the abort flag or because `limit_ns` passed since
// `start` (then the timeout is recorded with `where`).
static __device__ __noinline__ bool wait_expired(Ctrl *ctrl, uint64_t start, uint64_t limit_ns, int where) {
  if (ld_volatile_int(&ctrl->abort)) return true;
  if (globaltimer_ns() - start > limit_ns) {
    raise_error(ctrl, kErrTimeout, where);
    return true;
  }
  return false;
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
      ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive_count(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that lets the hardware suspend the thread until the phase
// completes or `hint_ns` passes, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with `parity` to complete.  Returns false on
// timeout or when another CTA raised the abort flag.  The first test is
// inline; a phase still open goes to the out-of-line loop.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t *bar, uint32_t parity, Ctrl *ctrl, uint64_t limit_ns,
                                            int where) {
  const uint64_t start = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, 20000u)) return true;
    if (wait_expired(ctrl, start, limit_ns, where)) return false;
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, Ctrl *ctrl,
                                          uint64_t limit_ns, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, ctrl, limit_ns, where);
}

// 16-byte asynchronous copy global -> shared (L2 only, no L1 allocation),
// grouped with cp_async_commit and completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Untiled bulk copy global -> shared, completion signalled on `bar`
// (16-byte aligned addresses, size a multiple of 16).  No multicast.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 evict-first policy: streamed weights are read once per step.
__device__ __forceinline__ void bulk_g2s_evict_first(void *smem_dst, const void *gmem_src,
                                                     uint32_t bytes, uint64_t *bar,
                                                     uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bulk prefetch of [src, src+bytes) into L2 (no completion tracking).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier over the consumer warps only (barrier 1); the producer warp
// never joins it.
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// ------------------------------------------------------------ grid barrier --
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int *p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add(unsigned int *p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// All CTAs of a cooperative launch: the consumer threads of each CTA sync,
// one thread publishes the CTA's writes and waits (bounded) until `target`
// arrivals are visible.  Returns false on timeout / abort.
__device__ __forceinline__ bool grid_barrier(Ctrl *ctrl, unsigned int target, int nthreads,
                                             uint64_t limit_ns, int *s_flag) {
  consumer_sync(nthreads);
  if (threadIdx.x == 0) {
    __threadfence();
    red_release_add(&ctrl->bar, 1u);
    int ok = 1;
    if (static_cast<int>(ld_acquire_u32(&ctrl->bar) - target) < 0) {
      const uint64_t start = globaltimer_ns();
      uint32_t spins = 0;
      while (static_cast<int>(ld_acquire_u32(&ctrl->bar) - target) < 0) {
        if ((++spins & 15u) == 0 && wait_expired(ctrl, start, limit_ns, kWhereGrid)) {
          ok = 0;
          break;
        }
      }
    }
    *s_flag = ok;
  }
  consumer_sync(nthreads);
  return *s_flag != 0;
}

// Test hook: wait on a flag nothing sets until the limit passes.
__device__ __forceinline__ void stall_on_unset_flag(Ctrl *ctrl, uint64_t limit_ns) {
  const uint64_t start = globaltimer_ns();
  while (ld_volatile_int(&ctrl->stall_flag) == 0) {
    if (ld_volatile_int(&ctrl->abort)) return;
    if (globaltimer_ns() - start > limit_ns) {
      raise_error(ctrl, kErrTimeout, kWhereStall);
      return;
    }
    __nanosleep(1000);
  }
}

// ------------------------------------------------------------ arithmetic --
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }
// Round to BF16 and back: the oracle's rounding points.
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// 8 BF16 weights x 8 BF16 activations, FP32 accumulate (two independent
// chains, summed at the end).
__device__ __forceinline__ float dot8_bf16(const uint4 w, const uint4 x, float acc) {
  float a = fmaf(bf_lo(w.x), bf_lo(x.x), acc);
  float b = bf_hi(w.x) * bf_hi(x.x);
  a = fmaf(bf_lo(w.y), bf_lo(x.y), a);
  b = fmaf(bf_hi(w.y), bf_hi(x.y), b);
  a = fmaf(bf_lo(w.z), bf_lo(x.z), a);
  b = fmaf(bf_hi(w.z), bf_hi(x.z), b);
  a = fmaf(bf_lo(w.w), bf_lo(x.w), a);
  b = fmaf(bf_hi(w.w), bf_hi(x.w), b);
  return a + b;
}

// Exact int8 -> FP32 for byte k of a word: build the float 2^23 + (b + 128)
// from the bits and subtract 2^23 + 128.
__device__ __forceinline__ float i8f(uint32_t biased_word, uint32_t selector) {
  return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, selector)) - 8388736.0f;
}

// 4 int8 weights (one word) x 4 BF16 activations (two words).
__device__ __forceinline__ float dot4_i8(uint32_t w, uint32_t x01, uint32_t x23, float acc) {
  const uint32_t b = w ^ 0x80808080u;
  float a0 = fmaf(i8f(b, 0x7540u), bf_lo(x01), acc);
  float a1 = i8f(b, 0x7541u) * bf_hi(x01);
  a0 = fmaf(i8f(b, 0x7542u), bf_lo(x23), a0);
  a1 = fmaf(i8f(b, 0x7543u), bf_hi(x23), a1);
  return a0 + a1;
}

// 16 int8 weights x 16 BF16 activations (x0: elements 0-7, x1: 8-15).
__device__ __forceinline__ float dot16_i8(const uint4 w, const uint4 x0, const uint4 x1,
                                          float acc) {
  const float a = dot4_i8(w.x, x0.x, x0.y, acc) + dot4_i8(w.y, x0.z, x0.w, 0.f);
  const float b = dot4_i8(w.z, x1.x, x1.y, 0.f) + dot4_i8(w.w, x1.z, x1.w, 0.f);
  return a + b;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Selection order of np.argmax (generate.py:713): a NaN ranks above every
// number, and among equal values (or NaNs) the lower index wins.  So the
// selected index is always one that was offered, whatever the values.
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
  const bool vn = isnan(v), bn = isnan(bv);
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

// (value, index) argmax merge in that order.
__device__ __forceinline__ void argmax_merge(float &v, int &i, float ov, int oi) {
  if (argmax_better(ov, oi, v, i)) {
    v = ov;
    i = oi;
  }
}

}  // namespace hb

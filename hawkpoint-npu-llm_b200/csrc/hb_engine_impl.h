// hb_engine_impl.h -- private to libhawkb200.so: the engine object and the
// host helpers shared by hb_engine.cu (persistent decoder path) and
// hb_batch.cu (batched tensor-core path).  Not part of the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "hawkb200.h"
#include "hb_decoder.cuh"

using hb::DecParams;
using hb::kMaxBatch;

namespace hbi {

constexpr uint64_t kDefaultLimitNs = 2000000000ull;  // 2 s per device wait
constexpr int kMaxSlotsRing = 16;
constexpr int kMinSlotsRing = 2;
// Pinned StepState staging buffers: one per upload within one call (a call
// may queue several launches before it synchronizes).
constexpr int kStateRing = 16;
constexpr int kProfileCap = 1 << 16;

extern thread_local std::string g_lib_error;

struct Variant {
  const void *fn = nullptr;
  size_t smem = 0;
  int nslots = 0;
  int mb = 0;
};

}  // namespace hbi

struct hb_sampler;
struct hb_batch;  // batched tensor-core path (hb_batch.cu), created on first use

struct hb_engine {
  int device = 0;
  hb_sampler *sampler = nullptr;  // created by the first hb_sample
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  hb_model_desc desc{};
  int G = 0;
  int red_rows = 0;
  int xs_elems = 0;
  hbi::Variant var1, var8;
  bool loaded = false;

  uint8_t *d_blob = nullptr;
  hb::LayerPtrs *d_layers = nullptr;
  float *d_rope_cos = nullptr, *d_rope_sin = nullptr;
  __nv_bfloat16 *d_kv = nullptr;
  size_t kv_slot_elems = 0;
  // paged KV cache (context > 64): pages of 64 positions, a page table per
  // slot (host copy authoritative, uploaded before a launch that follows a
  // change), reference counts for pages shared by copy_prefix
  bool paged = false;
  int pages_per_slot = 0, n_pages = 0;
  size_t page_bytes = 0;
  std::vector<int> page_table, page_refs, free_pages;
  bool table_dirty = false;
  int *d_page_table = nullptr;
  float *d_att_part = nullptr;
  int *d_att_cnt = nullptr;
  uint64_t *d_ll = nullptr;
  size_t ll_words = 0;
  unsigned int *d_epoch = nullptr;
  float *d_logits = nullptr, *d_part_val = nullptr;
  int *d_part_idx = nullptr;
  hb::Result *d_result = nullptr;
  hb::StepState *d_st = nullptr;
  int *d_prompt = nullptr, *d_gen = nullptr;
  unsigned long long *d_trace = nullptr;

  hb::StepState *h_st = nullptr;
  hb::Result *h_result = nullptr;
  int *h_prompt = nullptr, *h_gen = nullptr;

  std::vector<hb::LayerPtrs> layer_ptrs;
  std::string last_error;
  uint64_t limit_ns = hbi::kDefaultLimitNs;
  hb_batch *batch = nullptr;
  uint64_t stall_next_ns = 0;
  bool trace_enabled = false;

  bool profiling = false;
  std::vector<cudaEvent_t> ev_a, ev_b;
  int prof_count = 0;
};

namespace hbi {

inline int fail(hb_engine *e, int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (e) e->last_error = buf;
  g_lib_error = buf;
  return code;
}

#define HB_CUDA(e, call)                                                              \
  do {                                                                                \
    cudaError_t err_ = (call);                                                        \
    if (err_ != cudaSuccess)                                                          \
      return fail((e), HB_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(err_));       \
  } while (0)

// Makes the engine's device current for one call and restores the caller's
// current device on return, so the library never changes it behind the
// caller's back.
struct DeviceScope {
  int prev = -1;
  bool ok = false;
  explicit DeviceScope(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    ok = cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
#define HB_ON_DEVICE(e)                                                               \
  DeviceScope device_scope_((e)->device);                                            \
  if (!device_scope_.ok) return fail((e), HB_ERR_CUDA, "cudaSetDevice(%d) failed", (e)->device)

template <class T>
int dev_alloc(hb_engine *e, T **p, size_t count) {
  HB_CUDA(e, cudaMalloc(reinterpret_cast<void **>(p), sizeof(T) * (count ? count : 1)));
  HB_CUDA(e, cudaMemset(*p, 0, sizeof(T) * (count ? count : 1)));
  return HB_OK;
}

// Frees the batched tensor-core path's buffers (hb_batch.cu).
void batch_release(hb_engine *e);

}  // namespace hbi


// hb_engine.cu -- host side of libhawkb200.so (C ABI in include/hawkb200.h).
//
// Owns the device buffers of one engine (weights blob, per-slot KV cache,
// step activations, control block), launches the persistent decoder kernel
// cooperatively (all CTAs co-resident, one per SM, so the grid barriers always
// complete), reads back one small result block per call and turns device-side
// wait timeouts into HB_ERR_DEVICE_TIMEOUT.
#include <atomic>

#include "hb_engine_impl.h"
#include "hb_gemv.cuh"
#include "hb_sample.cuh"

using hb::DecParams;
using hb::kMaxBatch;
using namespace hbi;

thread_local std::string hbi::g_lib_error;

namespace {

int validate_desc(const hb_model_desc *d) {
  if (!d) return fail(nullptr, HB_ERR_INVALID_ARG, "desc is NULL");
  if (d->abi_version != HB_ABI_VERSION)
    return fail(nullptr, HB_ERR_INVALID_ARG, "abi_version %d != %d", d->abi_version, HB_ABI_VERSION);
  if (d->head_dim != hb::kHeadDim) return fail(nullptr, HB_ERR_UNSUPPORTED, "head_dim must be 64");
  if (d->hidden <= 0 || d->intermediate <= 0 || d->q_heads <= 0 || d->kv_heads <= 0 ||
      d->layers <= 0 || d->vocab <= 0 || d->context <= 0)
    return fail(nullptr, HB_ERR_INVALID_ARG, "invalid model dimensions");
  if (d->q_heads % d->kv_heads) return fail(nullptr, HB_ERR_INVALID_ARG, "q_heads %% kv_heads != 0");
  if (d->hidden != d->q_heads * d->head_dim)
    return fail(nullptr, HB_ERR_UNSUPPORTED, "hidden must equal q_heads * head_dim");
  if (d->weight_format != HB_WEIGHTS_BF16 && d->weight_format != HB_WEIGHTS_W8)
    return fail(nullptr, HB_ERR_INVALID_ARG, "unknown weight_format");
  const int qkv = (d->q_heads + 2 * d->kv_heads) * d->head_dim;
  if (d->hidden % 16 || d->intermediate % 16 || qkv % 8 || d->vocab % 8)
    return fail(nullptr, HB_ERR_UNSUPPORTED, "dimensions must be multiples of 16 (rows of 8)");
  const int esize = d->weight_format == HB_WEIGHTS_W8 ? 1 : 2;
  if (d->hidden * esize > 2048)
    return fail(nullptr, HB_ERR_UNSUPPORTED, "hidden too large for one LM-head chunk");
  if (d->hidden > hb::kMaxHPerThread * hb::kConsumerThreads)
    return fail(nullptr, HB_ERR_UNSUPPORTED, "hidden > %d", hb::kMaxHPerThread * hb::kConsumerThreads);
  // attention: 8-position tiles of a 64-position context, split over at
  // least two warps per kv head; longer contexts use 64-position pages
  if (d->kv_heads > 4) return fail(nullptr, HB_ERR_UNSUPPORTED, "kv_heads <= 4 required");
  if (d->context > hb::kPagePositions &&
      (d->context % hb::kPagePositions || d->context > hb::kMaxPagedContext))
    return fail(nullptr, HB_ERR_UNSUPPORTED, "context must be <= 64, or a multiple of 64 up to %d",
                hb::kMaxPagedContext);
  if (d->max_slots <= 0 || d->max_batch <= 0 || d->max_batch > kMaxBatch)
    return fail(nullptr, HB_ERR_INVALID_ARG, "max_slots > 0 and 1 <= max_batch <= 8 required");
  if (!d->layer_offsets || !d->rope_cos || !d->rope_sin)
    return fail(nullptr, HB_ERR_INVALID_ARG, "layer_offsets / rope tables missing");
  // every tensor inside the blob and 16-byte aligned (bulk copies need it)
  const uint64_t B = d->blob_bytes;
  auto in_blob = [&](uint64_t off, uint64_t bytes) { return off % 16 == 0 && off + bytes <= B; };
  const uint64_t h = d->hidden, I = d->intermediate;
  for (int l = 0; l < d->layers; ++l) {
    const hb_layer_offsets &o = d->layer_offsets[l];
    bool ok = in_blob(o.gamma_in, 4 * h) && in_blob(o.gamma_post, 4 * h) && in_blob(o.qkv_bias, 4 * qkv) &&
              in_blob(o.w_qkv, qkv * h * esize) && in_blob(o.w_o, h * h * esize) &&
              in_blob(o.w_gate_up, 2 * I * h * esize) && in_blob(o.w_down, h * I * esize);
    if (esize == 1)
      ok = ok && in_blob(o.s_qkv, 4 * qkv) && in_blob(o.s_o, 4 * h) && in_blob(o.s_gate_up, 8 * I) &&
           in_blob(o.s_down, 4 * h);
    if (!ok) return fail(nullptr, HB_ERR_INVALID_ARG, "layer %d offsets outside the blob or unaligned", l);
  }
  bool ok = in_blob(d->gamma_final, 4 * h) && in_blob(d->w_lm, uint64_t(d->vocab) * h * esize) &&
            in_blob(d->embedding, uint64_t(d->vocab) * h * 2);
  if (esize == 1) ok = ok && in_blob(d->s_lm, 4ull * d->vocab);
  if (!ok) return fail(nullptr, HB_ERR_INVALID_ARG, "global offsets outside the blob or unaligned");
  return HB_OK;
}

int setup_variant(hb_engine *e, Variant &v, int mb, const void *fn, int smem_optin) {
  const hb_model_desc &d = e->desc;
  const int qkv = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
  const hb::SmemPlan base =
      hb::smem_plan(0, mb, e->xs_elems, d.hidden, qkv, d.q_heads, d.kv_heads, e->red_rows, d.context, e->paged);
  int nslots = static_cast<int>((static_cast<size_t>(smem_optin) - base.total - 16 * kMaxSlotsRing) /
                                hb::kSlotBytes);
  if (nslots > kMaxSlotsRing) nslots = kMaxSlotsRing;
  if (nslots < kMinSlotsRing)
    return fail(e, HB_ERR_UNSUPPORTED, "model too large for the shared-memory plan (batch %d)", mb);
  const hb::SmemPlan sp =
      hb::smem_plan(nslots, mb, e->xs_elems, d.hidden, qkv, d.q_heads, d.kv_heads, e->red_rows, d.context, e->paged);
  HB_CUDA(e, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sp.total)));
  int blocks = 0;
  HB_CUDA(e, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, hb::kThreads, sp.total));
  if (blocks < 1) return fail(e, HB_ERR_UNSUPPORTED, "decoder kernel does not fit on an SM");
  v.fn = fn;
  v.smem = sp.total;
  v.nslots = nslots;
  v.mb = mb;
  return HB_OK;
}

DecParams base_params(hb_engine *e, const Variant &v) {
  const hb_model_desc &d = e->desc;
  const int esize = d.weight_format == HB_WEIGHTS_W8 ? 1 : 2;
  DecParams P{};
  P.H = d.hidden;
  P.I = d.intermediate;
  P.QH = d.q_heads;
  P.KVH = d.kv_heads;
  P.L = d.layers;
  P.V = d.vocab;
  P.CTX = d.context;
  P.QKV = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
  P.group = d.q_heads / d.kv_heads;
  P.has_bias = d.has_qkv_bias;
  P.eps = d.rms_eps;
  P.kc_h = d.hidden * esize / 16;
  P.kc_i = d.intermediate * esize / 16;
  P.layers = e->d_layers;
  P.gamma_final = reinterpret_cast<const float *>(e->d_blob + d.gamma_final);
  P.w_lm = e->d_blob + d.w_lm;
  P.s_lm = esize == 1 ? reinterpret_cast<const float *>(e->d_blob + d.s_lm) : nullptr;
  P.embed = reinterpret_cast<const __nv_bfloat16 *>(e->d_blob + d.embedding);
  P.rope_cos = e->d_rope_cos;
  P.rope_sin = e->d_rope_sin;
  P.kv = e->d_kv;
  P.ll = e->d_ll;
  P.epoch = e->d_epoch;
  P.logits = e->d_logits;
  P.part_val = e->d_part_val;
  P.part_idx = e->d_part_idx;
  P.result = e->d_result;
  P.st = e->d_st;
  P.prompt = e->d_prompt;
  P.gen_out = e->d_gen;
  P.red_rows = e->red_rows;
  P.nslots = v.nslots;
  P.xs_elems = e->xs_elems;
  P.limit_ns = e->limit_ns;
  P.trace = e->trace_enabled ? e->d_trace : nullptr;
  P.paged = e->paged ? 1 : 0;
  P.pages_per_slot = e->pages_per_slot;
  P.n_pages = e->n_pages;
  P.page_table = e->d_page_table;
  P.att_part = e->d_att_part;
  P.att_cnt = e->d_att_cnt;
  return P;
}

template <bool PG>
const void *decoder_fn_t(int mb, bool w8) {
  if (mb == 1) return w8 ? reinterpret_cast<const void *>(&hb::decoder_kernel<1, true, PG>)
                         : reinterpret_cast<const void *>(&hb::decoder_kernel<1, false, PG>);
  return w8 ? reinterpret_cast<const void *>(&hb::decoder_kernel<8, true, PG>)
            : reinterpret_cast<const void *>(&hb::decoder_kernel<8, false, PG>);
}

// The kernels of a paged cache (context > 64) are separate instances, so
// the attention of the 64-position kernels compiles as it would alone.
const void *decoder_fn(int mb, bool w8, bool paged) {
  return paged ? decoder_fn_t<true>(mb, w8) : decoder_fn_t<false>(mb, w8);
}

// Launch phases [pb, pe) for the rows in d_st.
int launch(hb_engine *e, int rows, int pb, int pe, int write_logits) {
  const Variant &v = rows > 1 ? e->var8 : e->var1;
  DecParams P = base_params(e, v);
  P.phase_begin = pb;
  P.phase_end = pe;
  P.write_logits = write_logits;
  P.stall_ns = e->stall_next_ns;
  e->stall_next_ns = 0;
  void *args[] = {&P};
  const bool prof = e->profiling && e->prof_count < kProfileCap;
  if (prof) {
    while (static_cast<int>(e->ev_a.size()) <= e->prof_count) {
      cudaEvent_t a, b;
      HB_CUDA(e, cudaEventCreate(&a));
      HB_CUDA(e, cudaEventCreate(&b));
      e->ev_a.push_back(a);
      e->ev_b.push_back(b);
    }
    HB_CUDA(e, cudaEventRecord(e->ev_a[e->prof_count], e->stream));
  }
  HB_CUDA(e, cudaLaunchCooperativeKernel(v.fn, dim3(e->G), dim3(hb::kThreads), args, v.smem, e->stream));
  if (prof) {
    HB_CUDA(e, cudaEventRecord(e->ev_b[e->prof_count], e->stream));
    ++e->prof_count;
  }
  return HB_OK;
}

// Copies the result block back, waits, and maps a device error to a code.
int finish(hb_engine *e) {
  HB_CUDA(e, cudaMemcpyAsync(e->h_result, e->d_result, sizeof(hb::Result), cudaMemcpyDeviceToHost, e->stream));
  HB_CUDA(e, cudaStreamSynchronize(e->stream));
  if (e->h_result->ctrl.err != 0) {
    const int code = e->h_result->ctrl.err;
    const int where = e->h_result->ctrl.err_where;
    // words of the aborted launch may carry the current epoch: clear them all
    HB_CUDA(e, cudaMemsetAsync(e->d_ll, 0, e->ll_words * 8, e->stream));
    HB_CUDA(e, cudaMemsetAsync(e->d_result, 0, sizeof(hb::Result), e->stream));
    if (e->d_att_cnt)
      HB_CUDA(e, cudaMemsetAsync(e->d_att_cnt, 0, sizeof(int) * kMaxBatch * e->desc.q_heads, e->stream));
    HB_CUDA(e, cudaStreamSynchronize(e->stream));
    if (code == hb::kErrBadToken)
      return fail(e, HB_ERR_STATE, "device-chained token id outside the vocabulary; engine state reset");
    if (code == hb::kErrBadPage)
      return fail(e, HB_ERR_STATE, "KV page-table entry outside the page pool; engine state reset");
    static const char *names[] = {"?", "weight chunk", "ring slot", "grid barrier", "test stall flag", "drain"};
    return fail(e, HB_ERR_DEVICE_TIMEOUT, "device wait on %s timed out; engine state reset",
                names[(where >= 0 && where <= 5) ? where : 0]);
  }
  return HB_OK;
}

int check_engine(hb_engine *e) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  if (!e->loaded) return fail(e, HB_ERR_STATE, "weights not loaded");
  HB_ON_DEVICE(e);
  return HB_OK;
}

int check_row(hb_engine *e, int slot, int token, int position) {
  const hb_model_desc &d = e->desc;
  if (slot < 0 || slot >= d.max_slots) return fail(e, HB_ERR_INVALID_ARG, "slot %d outside [0, %d)", slot, d.max_slots);
  if (token < 0 || token >= d.vocab) return fail(e, HB_ERR_INVALID_ARG, "token id %d outside the vocabulary", token);
  if (position < 0 || position >= d.context)
    return fail(e, HB_ERR_INVALID_ARG, "position outside the %d-token context", d.context);
  return HB_OK;
}

// ---- paged KV cache -------------------------------------------------------------
uint8_t *page_ptr(hb_engine *e, int pg) { return reinterpret_cast<uint8_t *>(e->d_kv) + e->page_bytes * pg; }

// A page from the pool, zero-filled (a fresh slot reads zeros, as after a
// reset), with one reference.
int page_alloc(hb_engine *e, int *out) {
  if (e->free_pages.empty()) return fail(e, HB_ERR_STATE, "KV page pool exhausted");
  const int pg = e->free_pages.back();
  e->free_pages.pop_back();
  HB_CUDA(e, cudaMemsetAsync(page_ptr(e, pg), 0, e->page_bytes, e->stream));
  e->page_refs[pg] = 1;
  *out = pg;
  return HB_OK;
}

void page_release(hb_engine *e, int pg) {
  if (pg >= 0 && --e->page_refs[pg] == 0) e->free_pages.push_back(pg);
}

// Before a launch that reads positions [0, last] of a slot and writes
// positions [first_write, last]: every page up to last mapped, and every
// page written private (a page shared by copy_prefix is copied first).
int pages_for_step(hb_engine *e, int slot, int first_write, int last) {
  if (!e->paged) return HB_OK;
  int *row = e->page_table.data() + static_cast<size_t>(slot) * e->pages_per_slot;
  for (int i = 0; i <= last / hb::kPagePositions; ++i) {
    const int pg = row[i];
    if (pg < 0) {
      int rc = page_alloc(e, &row[i]);
      if (rc) return rc;
      e->table_dirty = true;
    } else if (i >= first_write / hb::kPagePositions && e->page_refs[pg] > 1) {
      int fresh = -1;
      int rc = page_alloc(e, &fresh);
      if (rc) return rc;
      HB_CUDA(e, cudaMemcpyAsync(page_ptr(e, fresh), page_ptr(e, pg), e->page_bytes, cudaMemcpyDeviceToDevice,
                                 e->stream));
      page_release(e, pg);
      row[i] = fresh;
      e->table_dirty = true;
    }
  }
  return HB_OK;
}

// Uploads the page table after a change (from pageable memory: the copy
// has taken the table's contents when the call returns).
int upload_pages(hb_engine *e) {
  if (!e->paged || !e->table_dirty) return HB_OK;
  HB_CUDA(e, cudaMemcpyAsync(e->d_page_table, e->page_table.data(), sizeof(int) * e->page_table.size(),
                             cudaMemcpyHostToDevice, e->stream));
  e->table_dirty = false;
  return HB_OK;
}

// Device-resident chained run: positions start..n_prompt-1 of ids (prefill;
// the LM head only at the last), then n_new-1 further greedy steps.
int run_chained(hb_engine *e, int slot, const int32_t *ids, int n_prompt, int start, int n_new,
                int32_t *out_tokens, float *last_logits) {
  const hb_model_desc &d = e->desc;
  if (!ids || n_prompt <= 0 || start < 0 || start >= n_prompt || n_new < 1)
    return fail(e, HB_ERR_INVALID_ARG, "invalid prompt range");
  if (n_prompt + n_new - 1 > d.context)
    return fail(e, HB_ERR_INVALID_ARG, "prompt + generated tokens exceed the %d-token context", d.context);
  for (int p = start; p < n_prompt; ++p) {
    int rc = check_row(e, slot, ids[p], p);
    if (rc) return rc;
  }
  for (int p = 0; p < d.context; ++p) e->h_prompt[p] = (p >= start && p < n_prompt) ? ids[p] : 0;
  // the chained launches write positions start .. n_prompt + n_new - 2
  int prc = pages_for_step(e, slot, start, n_prompt + n_new - 2);
  if (prc || (prc = upload_pages(e))) return prc;
  const int body = 4 * d.layers;
  const int full = 4 * d.layers + 1;
  int upload = 0;
  // the next pinned staging buffer; when all are taken, wait until the
  // queued copies have read them (long prompts need more launches than the
  // ring holds)
  auto next_state = [&](hb::StepState **out) -> int {
    if (upload == kStateRing) {
      HB_CUDA(e, cudaStreamSynchronize(e->stream));
      upload = 0;
    }
    *out = &e->h_st[upload++];
    return HB_OK;
  };
  int first = start;  // first position the chained (device-advanced) steps run
  if (d.max_batch > 1) {
    // batched prefill: up to kMaxBatch consecutive positions per launch, all
    // but the last prompt position (which the chained steps run with the head)
    for (int p0 = start; p0 < n_prompt - 1; p0 += kMaxBatch) {
      const int k = std::min(kMaxBatch, n_prompt - 1 - p0);
      hb::StepState *sbp = nullptr;
      if ((prc = next_state(&sbp))) return prc;
      hb::StepState &sb = *sbp;
      std::memset(&sb, 0, sizeof(sb));
      for (int i = 0; i < k; ++i) {
        sb.token[i] = ids[p0 + i];
        sb.pos[i] = p0 + i;
        sb.slot[i] = slot;
      }
      sb.rows = k;
      HB_CUDA(e, cudaMemcpyAsync(e->d_st, &sb, sizeof(hb::StepState), cudaMemcpyHostToDevice, e->stream));
      int rc = launch(e, k, 0, body, 0);
      if (rc) return rc;
    }
    first = n_prompt - 1;
  }
  hb::StepState *stp = nullptr;
  if ((prc = next_state(&stp))) return prc;
  hb::StepState &st = *stp;
  std::memset(&st, 0, sizeof(st));
  st.token[0] = ids[first];
  st.pos[0] = first;
  st.slot[0] = slot;
  st.rows = 1;
  st.chained = 1;
  st.n_prompt = n_prompt;
  st.n_out = 0;
  HB_CUDA(e, cudaMemcpyAsync(e->d_prompt, e->h_prompt, sizeof(int) * d.context, cudaMemcpyHostToDevice, e->stream));
  HB_CUDA(e, cudaMemcpyAsync(e->d_st, &st, sizeof(hb::StepState), cudaMemcpyHostToDevice, e->stream));
  for (int p = first; p < n_prompt - 1; ++p) {
    int rc = launch(e, 1, 0, body, 0);
    if (rc) return rc;
  }
  for (int t = 0; t < n_new; ++t) {
    const bool want_logits = last_logits != nullptr && t == n_new - 1;
    int rc = launch(e, 1, 0, full, want_logits ? 1 : 0);
    if (rc) return rc;
  }
  HB_CUDA(e, cudaMemcpyAsync(e->h_gen, e->d_gen, sizeof(int) * n_new, cudaMemcpyDeviceToHost, e->stream));
  if (last_logits)
    HB_CUDA(e, cudaMemcpyAsync(last_logits, e->d_logits, sizeof(float) * d.vocab, cudaMemcpyDeviceToHost, e->stream));
  int rc = finish(e);
  if (rc) return rc;
  if (out_tokens) std::memcpy(out_tokens, e->h_gen, sizeof(int) * n_new);
  return HB_OK;
}

}  // namespace

extern "C" {

int hb_device_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

const char *hb_library_error(void) { return g_lib_error.c_str(); }

const char *hb_last_error(const hb_engine *engine) {
  return engine ? engine->last_error.c_str() : g_lib_error.c_str();
}

int hb_create(const hb_model_desc *desc, int device, hb_engine **out) {
  if (!out) return fail(nullptr, HB_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  int rc = validate_desc(desc);
  if (rc) return rc;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return fail(nullptr, HB_ERR_INVALID_ARG, "CUDA device %d not available", device);
  }
  hb_engine *e = new hb_engine();
  e->device = device;
  e->desc = *desc;
  e->desc.layer_offsets = nullptr;
  e->desc.rope_cos = e->desc.rope_sin = nullptr;
  auto bail = [&](int code) {
    hb_destroy(e);
    return code;
  };
  DeviceScope device_scope_(device);
  if (!device_scope_.ok) return bail(fail(nullptr, HB_ERR_CUDA, "cudaSetDevice(%d) failed", device));
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
    return bail(fail(nullptr, HB_ERR_CUDA, "cudaGetDeviceProperties failed"));
  if (prop.major < 10) return bail(fail(nullptr, HB_ERR_UNSUPPORTED, "this build targets sm_100a (B200)"));
  if (!prop.cooperativeLaunch) return bail(fail(nullptr, HB_ERR_UNSUPPORTED, "cooperative launch unsupported"));
  const hb_model_desc &d = e->desc;
  e->G = prop.multiProcessorCount;
  // the attention phase gives each (batch row, q head) unit its own CTA
  if (e->G < d.q_heads * d.max_batch)
    return bail(fail(nullptr, HB_ERR_UNSUPPORTED, "q_heads * max_batch (%d) exceeds the SM count (%d)",
                     d.q_heads * d.max_batch, e->G));
  const int qkv = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
  auto ceil_div = [](int a, int b) { return (a + b - 1) / b; };
  e->red_rows = std::max(std::max(ceil_div(qkv / 8, e->G) * 8, ceil_div(d.intermediate / 8, e->G) * 16),
                         ceil_div(d.hidden / 8, e->G) * 8);
  e->xs_elems = std::max(d.hidden, d.intermediate);  // GEMV inputs
  e->xs_elems = (e->xs_elems + 15) / 16 * 16;
  const bool w8 = d.weight_format == HB_WEIGHTS_W8;
  const bool paged = d.context > hb::kPagePositions;
  e->paged = paged;  // sizes the attention scratch of the shared-memory plan
  if ((rc = setup_variant(e, e->var1, 1, decoder_fn(1, w8, paged), prop.sharedMemPerBlockOptin))) return bail(rc);
  if (d.max_batch > 1 &&
      (rc = setup_variant(e, e->var8, 8, decoder_fn(8, w8, paged), prop.sharedMemPerBlockOptin)))
    return bail(rc);
  if (cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(fail(nullptr, HB_ERR_CUDA, "stream creation failed"));
  e->stream = e->own_stream;

  const int mb = d.max_batch > 1 ? kMaxBatch : 1;
  e->kv_slot_elems = static_cast<size_t>(d.layers) * d.kv_heads * 2 * d.context * hb::kHeadDim;
  if (paged) {
    // every slot can reach the full context with private pages
    e->pages_per_slot = d.context / hb::kPagePositions;
    e->n_pages = d.max_slots * e->pages_per_slot;
    e->page_bytes = static_cast<size_t>(d.layers) * d.kv_heads * 2 * hb::kPagePositions * hb::kHeadDim * 2;
    e->page_table.assign(static_cast<size_t>(d.max_slots) * e->pages_per_slot, -1);
    e->page_refs.assign(e->n_pages, 0);
    for (int pg = e->n_pages - 1; pg >= 0; --pg) e->free_pages.push_back(pg);
    e->table_dirty = true;
    if ((rc = dev_alloc(e, &e->d_page_table, e->page_table.size())) ||
        (rc = dev_alloc(e, &e->d_att_part, static_cast<size_t>(e->G) * hb::kPartStride)) ||
        (rc = dev_alloc(e, &e->d_att_cnt, static_cast<size_t>(kMaxBatch) * d.q_heads)))
      return bail(rc);
  }
  e->ll_words = hb::ll_layer_words(d.hidden, d.intermediate, qkv) * d.layers;
  const size_t half = static_cast<size_t>(d.head_dim / 2) * d.context;
  if ((rc = dev_alloc(e, &e->d_blob, d.blob_bytes)) || (rc = dev_alloc(e, &e->d_layers, d.layers)) ||
      (rc = dev_alloc(e, &e->d_rope_cos, half)) || (rc = dev_alloc(e, &e->d_rope_sin, half)) ||
      (rc = dev_alloc(e, &e->d_kv, e->kv_slot_elems * d.max_slots)) ||
      (rc = dev_alloc(e, &e->d_ll, e->ll_words)) || (rc = dev_alloc(e, &e->d_epoch, 1)) ||
      (rc = dev_alloc(e, &e->d_logits, static_cast<size_t>(kMaxBatch) * d.vocab)) ||
      (rc = dev_alloc(e, &e->d_part_val, static_cast<size_t>(e->G) * kMaxBatch)) ||
      (rc = dev_alloc(e, &e->d_part_idx, static_cast<size_t>(e->G) * kMaxBatch)) ||
      (rc = dev_alloc(e, &e->d_result, 1)) || (rc = dev_alloc(e, &e->d_st, 1)) ||
      (rc = dev_alloc(e, &e->d_prompt, d.context)) || (rc = dev_alloc(e, &e->d_gen, d.context + 1)) ||
      (rc = dev_alloc(e, &e->d_trace, static_cast<size_t>(e->G) * (4 * d.layers + 2) * 8)))
    return bail(rc);
  (void)mb;
  if (cudaHostAlloc(reinterpret_cast<void **>(&e->h_st), sizeof(hb::StepState) * kStateRing,
                    cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&e->h_result), sizeof(hb::Result), cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&e->h_prompt), sizeof(int) * d.context, cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&e->h_gen), sizeof(int) * (d.context + 1), cudaHostAllocDefault) != cudaSuccess)
    return bail(fail(nullptr, HB_ERR_CUDA, "pinned host allocation failed"));

  // device pointers of every layer's tensors
  const bool has_scales = w8;
  e->layer_ptrs.resize(d.layers);
  for (int l = 0; l < d.layers; ++l) {
    const hb_layer_offsets &o = desc->layer_offsets[l];
    hb::LayerPtrs &p = e->layer_ptrs[l];
    auto f = [&](uint64_t off) { return reinterpret_cast<const float *>(e->d_blob + off); };
    p.gamma_in = f(o.gamma_in);
    p.gamma_post = f(o.gamma_post);
    p.bias = f(o.qkv_bias);
    p.w_qkv = e->d_blob + o.w_qkv;
    p.w_o = e->d_blob + o.w_o;
    p.w_gu = e->d_blob + o.w_gate_up;
    p.w_down = e->d_blob + o.w_down;
    p.s_qkv = has_scales ? f(o.s_qkv) : nullptr;
    p.s_o = has_scales ? f(o.s_o) : nullptr;
    p.s_gu = has_scales ? f(o.s_gate_up) : nullptr;
    p.s_down = has_scales ? f(o.s_down) : nullptr;
  }
  if (cudaMemcpy(e->d_layers, e->layer_ptrs.data(), sizeof(hb::LayerPtrs) * d.layers, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(e->d_rope_cos, desc->rope_cos, sizeof(float) * half, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(e->d_rope_sin, desc->rope_sin, sizeof(float) * half, cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(fail(nullptr, HB_ERR_CUDA, "descriptor upload failed"));
  const unsigned int first_epoch = 1;
  if (cudaMemcpy(e->d_epoch, &first_epoch, sizeof(first_epoch), cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(fail(nullptr, HB_ERR_CUDA, "epoch upload failed"));
  if ((rc = upload_pages(e))) return bail(rc);
  if (cudaStreamSynchronize(e->stream) != cudaSuccess)
    return bail(fail(nullptr, HB_ERR_CUDA, "page table upload failed"));
  *out = e;
  return HB_OK;
}

int hb_load_weights(hb_engine *e, const void *host_blob, size_t bytes, int layout_version) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  if (!host_blob || bytes != e->desc.blob_bytes)
    return fail(e, HB_ERR_INVALID_ARG, "blob size %zu != %llu", bytes,
                static_cast<unsigned long long>(e->desc.blob_bytes));
  if (layout_version != 1) return fail(e, HB_ERR_UNSUPPORTED, "layout version %d unsupported", layout_version);
  HB_ON_DEVICE(e);
  HB_CUDA(e, cudaMemcpy(e->d_blob, host_blob, bytes, cudaMemcpyHostToDevice));
  e->loaded = true;
  return HB_OK;
}

int hb_destroy(hb_engine *e) {
  if (!e) return HB_OK;
  DeviceScope device_scope_(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  batch_release(e);
  for (auto ev : e->ev_a) cudaEventDestroy(ev);
  for (auto ev : e->ev_b) cudaEventDestroy(ev);
  void *dev[] = {e->d_blob, e->d_layers, e->d_rope_cos, e->d_rope_sin, e->d_kv, e->d_ll, e->d_epoch,
                 e->d_logits, e->d_part_val, e->d_part_idx, e->d_result, e->d_st, e->d_prompt,
                 e->d_gen, e->d_trace, e->d_page_table, e->d_att_part, e->d_att_cnt};
  for (void *p : dev)
    if (p) cudaFree(p);
  void *host[] = {e->h_st, e->h_result, e->h_prompt, e->h_gen};
  for (void *p : host)
    if (p) cudaFreeHost(p);
  if (e->own_stream) cudaStreamDestroy(e->own_stream);
  hb_sampler *sampler = e->sampler;
  delete e;
  hb_sampler_destroy(sampler);
  return HB_OK;
}

int hb_step(hb_engine *e, int slot, int token_id, int position, int flags, float *logits_out,
            int32_t *argmax_out) {
  int rc = check_engine(e);
  if (rc) return rc;
  if ((rc = check_row(e, slot, token_id, position))) return rc;
  if ((rc = pages_for_step(e, slot, position, position)) || (rc = upload_pages(e))) return rc;
  if (logits_out) flags |= HB_STEP_LOGITS;
  if (flags & (HB_STEP_LOGITS | HB_STEP_DEVICE_LOGITS)) flags |= HB_STEP_ARGMAX;
  const int device_logits = (logits_out || (flags & HB_STEP_DEVICE_LOGITS)) ? 1 : 0;
  hb::StepState &st = *e->h_st;
  std::memset(&st, 0, sizeof(st));
  st.token[0] = token_id;
  st.pos[0] = position;
  st.slot[0] = slot;
  st.rows = 1;
  HB_CUDA(e, cudaMemcpyAsync(e->d_st, e->h_st, sizeof(hb::StepState), cudaMemcpyHostToDevice, e->stream));
  const int pe = (flags & HB_STEP_ARGMAX) ? 4 * e->desc.layers + 1 : 4 * e->desc.layers;
  if ((rc = launch(e, 1, 0, pe, device_logits))) return rc;
  if (logits_out)
    HB_CUDA(e, cudaMemcpyAsync(logits_out, e->d_logits, sizeof(float) * e->desc.vocab, cudaMemcpyDeviceToHost, e->stream));
  if ((rc = finish(e))) return rc;
  if (argmax_out) *argmax_out = (flags & HB_STEP_ARGMAX) ? e->h_result->out_token[0] : -1;
  return HB_OK;
}

int hb_prefill(hb_engine *e, int slot, const int32_t *ids, int n, int start_pos, float *last_logits,
               int32_t *argmax_out) {
  int rc = check_engine(e);
  if (rc) return rc;
  if (!ids || n <= 0) return fail(e, HB_ERR_INVALID_ARG, "empty prefill");
  if (start_pos < 0 || start_pos + n > e->desc.context)
    return fail(e, HB_ERR_INVALID_ARG, "position outside the %d-token context", e->desc.context);
  std::vector<int32_t> by_pos(start_pos + n, 0);
  for (int i = 0; i < n; ++i) by_pos[start_pos + i] = ids[i];
  int32_t tok = -1;
  rc = run_chained(e, slot, by_pos.data(), start_pos + n, start_pos, 1, &tok, last_logits);
  if (rc) return rc;
  if (argmax_out) *argmax_out = tok;
  return HB_OK;
}

int hb_generate(hb_engine *e, int slot, const int32_t *ids, int n_prompt, int start_pos, int n_new,
                int32_t *out_tokens) {
  int rc = check_engine(e);
  if (rc) return rc;
  return run_chained(e, slot, ids, n_prompt, start_pos, n_new, out_tokens, nullptr);
}

int hb_step_batch(hb_engine *e, int n, const int32_t *slots, const int32_t *token_ids,
                  const int32_t *positions, int flags, float *logits_out, int32_t *argmax_out) {
  int rc = check_engine(e);
  if (rc) return rc;
  if (n < 1 || n > e->desc.max_batch || !slots || !token_ids || !positions)
    return fail(e, HB_ERR_INVALID_ARG, "batch of %d rows outside [1, %d]", n, e->desc.max_batch);
  for (int i = 0; i < n; ++i) {
    if ((rc = check_row(e, slots[i], token_ids[i], positions[i]))) return rc;
    for (int j = 0; j < i; ++j)
      if (slots[j] == slots[i]) return fail(e, HB_ERR_INVALID_ARG, "slot %d appears twice in one batch", slots[i]);
  }
  for (int i = 0; i < n; ++i)
    if ((rc = pages_for_step(e, slots[i], positions[i], positions[i]))) return rc;
  if ((rc = upload_pages(e))) return rc;
  if (logits_out) flags |= HB_STEP_LOGITS;
  if (flags & (HB_STEP_LOGITS | HB_STEP_DEVICE_LOGITS)) flags |= HB_STEP_ARGMAX;
  const int device_logits = (logits_out || (flags & HB_STEP_DEVICE_LOGITS)) ? 1 : 0;
  hb::StepState &st = *e->h_st;
  std::memset(&st, 0, sizeof(st));
  for (int i = 0; i < n; ++i) {
    st.token[i] = token_ids[i];
    st.pos[i] = positions[i];
    st.slot[i] = slots[i];
  }
  st.rows = n;
  HB_CUDA(e, cudaMemcpyAsync(e->d_st, e->h_st, sizeof(hb::StepState), cudaMemcpyHostToDevice, e->stream));
  const int pe = (flags & HB_STEP_ARGMAX) ? 4 * e->desc.layers + 1 : 4 * e->desc.layers;
  if ((rc = launch(e, n, 0, pe, device_logits))) return rc;
  if (logits_out)
    HB_CUDA(e, cudaMemcpyAsync(logits_out, e->d_logits, sizeof(float) * e->desc.vocab * n, cudaMemcpyDeviceToHost, e->stream));
  if ((rc = finish(e))) return rc;
  if (argmax_out)
    for (int i = 0; i < n; ++i) argmax_out[i] = (flags & HB_STEP_ARGMAX) ? e->h_result->out_token[i] : -1;
  return HB_OK;
}

int hb_reset(hb_engine *e, int slot) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  if (slot < 0 || slot >= e->desc.max_slots) return fail(e, HB_ERR_INVALID_ARG, "slot %d out of range", slot);
  HB_ON_DEVICE(e);
  if (e->paged) {
    // the slot's pages go back to the pool; its next steps map zeroed pages
    int *row = e->page_table.data() + static_cast<size_t>(slot) * e->pages_per_slot;
    for (int i = 0; i < e->pages_per_slot; ++i) {
      if (row[i] >= 0) e->table_dirty = true;
      page_release(e, row[i]);
      row[i] = -1;
    }
    int rc = upload_pages(e);
    if (rc) return rc;
  } else {
    HB_CUDA(e, cudaMemsetAsync(e->d_kv + e->kv_slot_elems * slot, 0, e->kv_slot_elems * 2, e->stream));
  }
  HB_CUDA(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

int hb_copy_prefix(hb_engine *e, int src, int dst, int n_positions) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  const hb_model_desc &d = e->desc;
  if (src < 0 || src >= d.max_slots || dst < 0 || dst >= d.max_slots)
    return fail(e, HB_ERR_INVALID_ARG, "slot out of range");
  if (n_positions < 0 || n_positions > d.context) return fail(e, HB_ERR_INVALID_ARG, "n_positions out of range");
  if (src == dst || n_positions == 0) return HB_OK;
  HB_ON_DEVICE(e);
  if (e->paged) {
    // whole pages below n_positions are shared (copied on their next
    // write); the rows [0, n % 64) of a partial page are copied
    int *srow = e->page_table.data() + static_cast<size_t>(src) * e->pages_per_slot;
    int *drow = e->page_table.data() + static_cast<size_t>(dst) * e->pages_per_slot;
    const int full = n_positions / hb::kPagePositions, rem = n_positions % hb::kPagePositions;
    for (int i = 0; i < full; ++i) {
      if (drow[i] == srow[i]) continue;
      if (srow[i] >= 0) ++e->page_refs[srow[i]];
      page_release(e, drow[i]);
      drow[i] = srow[i];
      e->table_dirty = true;
    }
    if (rem) {
      int rc = pages_for_step(e, dst, full * hb::kPagePositions, full * hb::kPagePositions);
      if (rc) return rc;
      const size_t height = static_cast<size_t>(d.layers) * d.kv_heads * 2;
      const size_t pitch = static_cast<size_t>(hb::kPagePositions) * 128;
      uint8_t *to = page_ptr(e, drow[full]);
      if (srow[full] >= 0)
        HB_CUDA(e, cudaMemcpy2DAsync(to, pitch, page_ptr(e, srow[full]), pitch, static_cast<size_t>(rem) * 128,
                                     height, cudaMemcpyDeviceToDevice, e->stream));
      else
        HB_CUDA(e, cudaMemset2DAsync(to, pitch, 0, static_cast<size_t>(rem) * 128, height, e->stream));
    }
    int rc = upload_pages(e);
    if (rc) return rc;
    HB_CUDA(e, cudaStreamSynchronize(e->stream));
    return HB_OK;
  }
  // every K and V block is [context][64] with 128-byte position rows: copy
  // the first n rows of each block
  const size_t pitch = static_cast<size_t>(d.context) * hb::kHeadDim * 2;
  const size_t height = static_cast<size_t>(d.layers) * d.kv_heads * 2;
  HB_CUDA(e, cudaMemcpy2DAsync(e->d_kv + e->kv_slot_elems * dst, pitch, e->d_kv + e->kv_slot_elems * src, pitch,
                               static_cast<size_t>(n_positions) * hb::kHeadDim * 2, height,
                               cudaMemcpyDeviceToDevice, e->stream));
  HB_CUDA(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

int hb_debug_dump(hb_engine *e, int what, void *out, size_t bytes) {
  if (!e || !out) return fail(e, HB_ERR_INVALID_ARG, "engine or out is NULL");
  HB_ON_DEVICE(e);
  const hb_model_desc &d = e->desc;
  if (what == HB_DUMP_HIDDEN) {
    // payloads of the last layer's output words: BF16 [kMaxBatch][hidden]
    const size_t need = static_cast<size_t>(kMaxBatch) * d.hidden * 2;
    if (bytes < need) return fail(e, HB_ERR_INVALID_ARG, "need %zu bytes", need);
    const int qkv = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
    const size_t lw = hb::ll_layer_words(d.hidden, d.intermediate, qkv);
    const size_t off = lw * (d.layers - 1) + static_cast<size_t>(kMaxBatch) * (qkv + d.hidden + d.intermediate) / 2;
    std::vector<uint64_t> words(static_cast<size_t>(kMaxBatch) * d.hidden / 2);
    HB_CUDA(e, cudaMemcpyAsync(words.data(), e->d_ll + off, words.size() * 8, cudaMemcpyDeviceToHost, e->stream));
    HB_CUDA(e, cudaStreamSynchronize(e->stream));
    uint32_t *o = static_cast<uint32_t *>(out);
    for (size_t i = 0; i < words.size(); ++i) o[i] = static_cast<uint32_t>(words[i]);
  } else if (what == HB_DUMP_KV) {
    const int slot = *reinterpret_cast<int *>(out);
    if (slot < 0 || slot >= d.max_slots) return fail(e, HB_ERR_INVALID_ARG, "slot out of range");
    const size_t need = e->kv_slot_elems * 2;
    if (bytes < need) return fail(e, HB_ERR_INVALID_ARG, "need %zu bytes", need);
    if (e->paged) {
      // gather the slot's pages into the [context][64] layout of each block
      const size_t blocks = static_cast<size_t>(d.layers) * d.kv_heads * 2;
      const size_t pitch = static_cast<size_t>(hb::kPagePositions) * 128, dpitch = static_cast<size_t>(d.context) * 128;
      uint8_t *o = static_cast<uint8_t *>(out);
      const int *row = e->page_table.data() + static_cast<size_t>(slot) * e->pages_per_slot;
      for (int i = 0; i < e->pages_per_slot; ++i) {
        if (row[i] >= 0) {
          HB_CUDA(e, cudaMemcpy2DAsync(o + i * pitch, dpitch, page_ptr(e, row[i]), pitch, pitch, blocks,
                                       cudaMemcpyDeviceToHost, e->stream));
        } else {
          for (size_t b = 0; b < blocks; ++b) std::memset(o + b * dpitch + i * pitch, 0, pitch);
        }
      }
    } else {
      HB_CUDA(e, cudaMemcpyAsync(out, e->d_kv + e->kv_slot_elems * slot, need, cudaMemcpyDeviceToHost, e->stream));
    }
  } else if (what == 2) {
    // phase trace: [G][4L+2] globaltimer stamps of the last traced launch
    const size_t need = static_cast<size_t>(e->G) * (4 * d.layers + 2) * 8 * 8;
    if (bytes < need) return fail(e, HB_ERR_INVALID_ARG, "need %zu bytes", need);
    HB_CUDA(e, cudaMemcpyAsync(out, e->d_trace, need, cudaMemcpyDeviceToHost, e->stream));
  } else {
    return fail(e, HB_ERR_INVALID_ARG, "unknown dump kind %d", what);
  }
  HB_CUDA(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

int hb_profile(hb_engine *e, int enable) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  e->profiling = enable & 1;
  e->trace_enabled = (enable & 2) != 0;
  e->prof_count = 0;
  return HB_OK;
}

int hb_profile_read(hb_engine *e, float *ms, float *start_ms, int max, int *count) {
  if (!e || !count || !ms) return fail(e, HB_ERR_INVALID_ARG, "engine, ms or count is NULL");
  HB_ON_DEVICE(e);
  HB_CUDA(e, cudaStreamSynchronize(e->stream));
  const int n = std::min(max, e->prof_count);
  for (int i = 0; i < n; ++i) {
    HB_CUDA(e, cudaEventElapsedTime(&ms[i], e->ev_a[i], e->ev_b[i]));
    if (start_ms) HB_CUDA(e, cudaEventElapsedTime(&start_ms[i], e->ev_a[0], e->ev_a[i]));
  }
  *count = n;
  e->prof_count = 0;
  return HB_OK;
}

int hb_set_stream(hb_engine *e, void *stream) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  e->stream = stream ? static_cast<cudaStream_t>(stream) : e->own_stream;
  return HB_OK;
}

int hb_test_stall_next(hb_engine *e, uint64_t limit_ns) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  if (limit_ns == 0 || limit_ns > 10000000000ull) return fail(e, HB_ERR_INVALID_ARG, "limit must be in (0, 10 s]");
  e->stall_next_ns = limit_ns;
  return HB_OK;
}

// ------------------------------------------------------------------ GEMV --
}  // extern "C"

namespace {

// Per device: the SM count and opt-in shared memory, queried once, and the
// dynamic shared memory each GEMV kernel variant has been opted into, so a
// call sets the attribute only when it needs more than any call before (the
// attribute call and the queries cost more than a small GEMV's kernel).
struct GemvDevice {
  bool known = false;
  int sms = 0, optin = 0;
  int smem[4] = {0, 0, 0, 0};  // by variant: (batch 8) * 2 + W8
};
constexpr int kGemvDevices = 64;
std::mutex g_gemv_mutex;
GemvDevice g_gemv_device[kGemvDevices];
// test hook (hb_test_gemv_stall_next): consumed by the next GEMV launch
std::atomic<uint64_t> g_gemv_stall_ns{0};

int gemv_device(int *dev, int *sms, int *optin) {
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= kGemvDevices)
    return fail(nullptr, HB_ERR_CUDA, "hb_gemv: no usable current CUDA device");
  std::lock_guard<std::mutex> lock(g_gemv_mutex);
  GemvDevice &g = g_gemv_device[*dev];
  if (!g.known) {
    if (cudaDeviceGetAttribute(&g.sms, cudaDevAttrMultiProcessorCount, *dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&g.optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, *dev) != cudaSuccess)
      return fail(nullptr, HB_ERR_CUDA, "hb_gemv: device query failed");
    g.known = true;
  }
  *sms = g.sms;
  *optin = g.optin;
  return HB_OK;
}

// Opts variant `v` (kernel fn) into `smem` bytes unless it already is;
// forget=true drops the record first (a launch that failed after a device
// reset lost the attribute).
int gemv_opt_in(int dev, int v, const void *fn, size_t smem, bool forget) {
  std::lock_guard<std::mutex> lock(g_gemv_mutex);
  int &have = g_gemv_device[dev].smem[v];
  if (forget) have = 0;
  if (have >= static_cast<int>(smem)) return HB_OK;
  const cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return fail(nullptr, HB_ERR_CUDA, "hb_gemv: %s", cudaGetErrorString(err));
  have = static_cast<int>(smem);
  return HB_OK;
}

// The GEMV kernel of (batch rows mb, W8) and its variant index.
const void *gemv_fn(int mb, bool w8, int *v) {
  *v = (mb > 1 ? 2 : 0) + (w8 ? 1 : 0);
  if (mb == 1)
    return w8 ? reinterpret_cast<const void *>(&hb::gemv_kernel<1, true>)
              : reinterpret_cast<const void *>(&hb::gemv_kernel<1, false>);
  return w8 ? reinterpret_cast<const void *>(&hb::gemv_kernel<8, true>)
            : reinterpret_cast<const void *>(&hb::gemv_kernel<8, false>);
}

// Launches a GEMV, retrying once with the attribute set again if the launch
// fails (the device was reset since the attribute was recorded).
int gemv_launch(int dev, int mb, bool w8, int grid, size_t smem, hb::GemvParams &P, cudaStream_t stream,
                const char *who) {
  int v = 0;
  const void *fn = gemv_fn(mb, w8, &v);
  P.stall_ns = g_gemv_stall_ns.exchange(0);
  int rc = gemv_opt_in(dev, v, fn, smem, false);
  if (rc) return rc;
  void *args[] = {&P};
  cudaError_t err = cudaLaunchKernel(fn, dim3(grid), dim3(hb::kThreads), args, smem, stream);
  if (err != cudaSuccess) {
    cudaGetLastError();
    if ((rc = gemv_opt_in(dev, v, fn, smem, true))) return rc;
    err = cudaLaunchKernel(fn, dim3(grid), dim3(hb::kThreads), args, smem, stream);
  }
  if (err != cudaSuccess) return fail(nullptr, HB_ERR_CUDA, "%s launch: %s", who, cudaGetErrorString(err));
  return HB_OK;
}

}  // namespace

extern "C" {

int hb_test_gemv_stall_next(uint64_t limit_ns) {
  if (limit_ns == 0 || limit_ns > 10000000000ull) return fail(nullptr, HB_ERR_INVALID_ARG, "limit must be in (0, 10 s]");
  g_gemv_stall_ns.store(limit_ns);
  return HB_OK;
}

size_t hb_gemv_scratch_bytes(int rows, int batch) {
  (void)rows;
  (void)batch;
  return sizeof(hb::Ctrl) + 2 * sizeof(float) * 1024 * hb::kMaxBatchGemv;
}

int hb_gemv(const void *w_dev, const float *scales_dev, int weight_format, int rows, int k, const void *x_dev,
            int batch, void *y_dev, int flags, int32_t *argmax_dev, void *scratch_dev, size_t scratch_bytes,
            void *stream) {
  const int out_mode = flags & 3;
  const bool want_argmax = (flags & HB_GEMV_ARGMAX) != 0;
  if (!w_dev || !x_dev || rows <= 0 || k <= 0 || rows % 8 || k % 32 || batch < 1 || batch > hb::kMaxBatchGemv)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_gemv: bad shape (rows %% 8, k %% 32, batch 1..8)");
  if (weight_format != HB_WEIGHTS_BF16 && weight_format != HB_WEIGHTS_W8)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_gemv: unknown weight format");
  if (weight_format == HB_WEIGHTS_W8 && !scales_dev) return fail(nullptr, HB_ERR_INVALID_ARG, "hb_gemv: W8 needs scales");
  if (out_mode > 2 || (out_mode != 2 && !y_dev)) return fail(nullptr, HB_ERR_INVALID_ARG, "hb_gemv: bad output");
  if (want_argmax && !argmax_dev) return fail(nullptr, HB_ERR_INVALID_ARG, "hb_gemv: argmax output missing");
  if (!scratch_dev || scratch_bytes < hb_gemv_scratch_bytes(rows, batch))
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_gemv: scratch too small");
  const auto check = [](uintptr_t p) { return p % 16 == 0; };
  if (!check(reinterpret_cast<uintptr_t>(w_dev)) || !check(reinterpret_cast<uintptr_t>(x_dev)))
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_gemv: W and x must be 16-byte aligned");
  int dev = 0, sms = 0, optin = 0;
  int rc = gemv_device(&dev, &sms, &optin);
  if (rc) return rc;
  const bool w8 = weight_format == HB_WEIGHTS_W8;
  const int esize = w8 ? 1 : 2;
  const int kc = k * esize / 16;
  const int n_rg = rows / 8;
  const int G = std::min(sms, n_rg);
  if (G > 1024) return fail(nullptr, HB_ERR_UNSUPPORTED, "hb_gemv: too many SMs");
  const int rg_per_cta = (n_rg + G - 1) / G;
  const bool whole = kc * 128 <= static_cast<int>(hb::kSlotBytes);
  const int per_warp = (whole && rg_per_cta >= 16) ? 1 : 0;
  const int red_rows = per_warp ? 1 : rg_per_cta * 8;
  const int mb = batch > 1 ? 8 : 1;
  const size_t fixed = hb::gemv_smem_bytes(0, mb, k, red_rows);
  // (checked before subtracting: the sizes are unsigned)
  if (fixed + 16 * kMaxSlotsRing + static_cast<size_t>(kMinSlotsRing) * hb::kSlotBytes > static_cast<size_t>(optin))
    return fail(nullptr, HB_ERR_UNSUPPORTED, "hb_gemv: shape too large for shared memory");
  int nslots = static_cast<int>((static_cast<size_t>(optin) - fixed - 16 * kMaxSlotsRing) / hb::kSlotBytes);
  nslots = std::min(nslots, kMaxSlotsRing);
  const size_t smem = hb::gemv_smem_bytes(nslots, mb, k, red_rows);
  hb::GemvParams P{};
  P.w = static_cast<const uint8_t *>(w_dev);
  P.scales = scales_dev;
  P.rows = rows;
  P.kc = kc;
  P.K = k;
  P.x = static_cast<const __nv_bfloat16 *>(x_dev);
  P.batch = batch;
  P.y = y_dev;
  P.out_mode = out_mode;
  P.argmax = want_argmax ? 1 : 0;
  P.argmax_out = argmax_dev;
  P.ctrl = static_cast<hb::Ctrl *>(scratch_dev);
  P.part_val = reinterpret_cast<float *>(static_cast<uint8_t *>(scratch_dev) + sizeof(hb::Ctrl));
  P.part_idx = reinterpret_cast<int *>(P.part_val + 1024 * hb::kMaxBatchGemv);
  P.nslots = nslots;
  P.red_rows = red_rows;
  P.per_warp = per_warp;
  P.limit_ns = kDefaultLimitNs;
  return gemv_launch(dev, mb, w8, G, smem, P, static_cast<cudaStream_t>(stream), "hb_gemv");
}

}  // extern "C"

// ------------------------------------------------------- hb_gemv_noalloc --
// The standalone GEMV (+ fused argmax) without a caller-supplied scratch
// buffer.
//
// hb_gemv needs a small device scratch area (a control block with the
// done-counter of the fused argmax and one partial (value, index) per CTA and
// batch row), and asks the caller to allocate it.  Some callers cannot: a
// serving process that sized its whole GPU memory pool (weights plus KV
// cache) at start-up and forbids device allocations afterwards, or a hot path
// that must not call cudaMalloc / cudaFree because those can synchronize the
// device and stall every other stream.  This section gives them a variant
// whose scratch lives in a fixed, file-scope __device__ array that the
// library owns.
//
// Limits and sharing rules:
// * the array holds kNoAllocCtas partial results per batch row for up to
//   kNoAllocBatch batch rows (65,568 bytes in all, control block included);
//   requests that would need more are rejected with HB_ERR_UNSUPPORTED;
// * every GPU that loads the library holds one copy of the array until the
//   process exits;
// * the first call on a device looks up the array's device address
//   (cudaGetSymbolAddress, with that device current) and caches it, so that
//   first call should come before any stream capture; the cached address
//   belongs to the device's primary context, so a process that calls
//   cudaDeviceReset after using this entry point must not call it again;
// * a device-side wait that gives up (HB_ERR_DEVICE_TIMEOUT on other entry
//   points) is reported in-band: the argmax of every batch row reads -1
//   (the control block lives in the array, which the caller cannot read);
// * all calls on a device share that one array, so calls whose kernels could
//   run at the same time on the GPU (different streams, no ordering between
//   them) race on it and may return wrong argmax results; order such calls
//   on one stream;
// * the array keeps whatever the previous call left in it, so each call
//   clears the control block (cudaMemsetAsync, no allocation) before its
//   launch.
// The entry point allocates nothing: no cudaMalloc, no cudaFree, no library
// routine that allocates.
namespace {

constexpr int kNoAllocCtas = 1024;                    // partial slots per batch row
constexpr int kNoAllocBatch = hb::kMaxBatchGemv;      // 8 batch rows
constexpr size_t kNoAllocScratchBytes =
    sizeof(hb::Ctrl) + 2 * sizeof(float) * kNoAllocCtas * kNoAllocBatch;  // 65,568 bytes
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a stand-in for the
// device symbol, never a device address: the device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_dev[kMaxDevices] = {};

int noalloc_fail(int code, const char *msg) { return fail(nullptr, code, "hb_gemv_noalloc: %s", msg); }

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) and cached.
int scratch_address(int device, void **out) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_dev[device] == nullptr) {
    void *ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return noalloc_fail(HB_ERR_CUDA, cudaGetErrorString(err));
    g_scratch_dev[device] = ptr;
  }
  *out = g_scratch_dev[device];
  return HB_OK;
}

}  // namespace

extern "C" {

int hb_gemv_noalloc(const void *w_dev, const float *scales_dev, int weight_format, int rows, int k,
                    const void *x_dev, int batch, void *y_dev, int flags, int32_t *argmax_dev,
                    void *stream) {
  const int out_mode = flags & 3;
  const bool want_argmax = (flags & HB_GEMV_ARGMAX) != 0;
  if (!w_dev || !x_dev || rows <= 0 || k <= 0 || rows % 8 || k % 32)
    return noalloc_fail(HB_ERR_INVALID_ARG, "bad shape (rows % 8 == 0 and k % 32 == 0 required)");
  if (batch < 1) return noalloc_fail(HB_ERR_INVALID_ARG, "batch must be at least 1");
  if (batch > kNoAllocBatch)
    return noalloc_fail(HB_ERR_UNSUPPORTED, "batch exceeds the 8 rows the built-in scratch holds");
  if (weight_format != HB_WEIGHTS_BF16 && weight_format != HB_WEIGHTS_W8)
    return noalloc_fail(HB_ERR_INVALID_ARG, "unknown weight format");
  if (weight_format == HB_WEIGHTS_W8 && !scales_dev)
    return noalloc_fail(HB_ERR_INVALID_ARG, "W8 weights need scales");
  if (out_mode > 2 || (out_mode != 2 && !y_dev)) return noalloc_fail(HB_ERR_INVALID_ARG, "bad output");
  if (want_argmax && !argmax_dev) return noalloc_fail(HB_ERR_INVALID_ARG, "argmax output missing");
  if (reinterpret_cast<uintptr_t>(w_dev) % 16 || reinterpret_cast<uintptr_t>(x_dev) % 16)
    return noalloc_fail(HB_ERR_INVALID_ARG, "W and x must be 16-byte aligned");

  int dev = 0, sms = 0, optin = 0;
  if (gemv_device(&dev, &sms, &optin) != HB_OK || dev >= kMaxDevices)
    return noalloc_fail(HB_ERR_CUDA, "no usable current CUDA device");
  const int n_rg = rows / 8;
  const int G = sms < n_rg ? sms : n_rg;
  // one CTA per SM at most: this only guards a future grid with more CTAs
  if (G > kNoAllocCtas)
    return noalloc_fail(HB_ERR_UNSUPPORTED, "more CTAs than the built-in scratch has partial slots");

  void *scratch = nullptr;
  int rc = scratch_address(dev, &scratch);
  if (rc != HB_OK) return rc;

  const bool w8 = weight_format == HB_WEIGHTS_W8;
  const int esize = w8 ? 1 : 2;
  const int kc = k * esize / 16;
  const int rg_per_cta = (n_rg + G - 1) / G;
  const bool whole = kc * 128 <= static_cast<int>(hb::kSlotBytes);
  const int per_warp = (whole && rg_per_cta >= 16) ? 1 : 0;
  const int red_rows = per_warp ? 1 : rg_per_cta * 8;
  const int mb = batch > 1 ? 8 : 1;
  const size_t fixed = hb::gemv_smem_bytes(0, mb, k, red_rows);
  // (checked before subtracting: the sizes are unsigned)
  if (fixed + 16 * 16 + 4 * static_cast<size_t>(hb::kSlotBytes) > static_cast<size_t>(optin))
    return noalloc_fail(HB_ERR_UNSUPPORTED, "shape too large for shared memory");
  int nslots = static_cast<int>((static_cast<size_t>(optin) - fixed - 16 * 16) / hb::kSlotBytes);
  if (nslots > 16) nslots = 16;
  const size_t smem = hb::gemv_smem_bytes(nslots, mb, k, red_rows);

  // the control block must start at zero (done counter, error flags)
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemsetAsync(scratch, 0, sizeof(hb::Ctrl), s);
  if (err != cudaSuccess) return noalloc_fail(HB_ERR_CUDA, cudaGetErrorString(err));

  hb::GemvParams P{};
  P.w = static_cast<const uint8_t *>(w_dev);
  P.scales = scales_dev;
  P.rows = rows;
  P.kc = kc;
  P.K = k;
  P.x = static_cast<const __nv_bfloat16 *>(x_dev);
  P.batch = batch;
  P.y = y_dev;
  P.out_mode = out_mode;
  P.argmax = want_argmax ? 1 : 0;
  P.argmax_out = argmax_dev;
  P.ctrl = static_cast<hb::Ctrl *>(scratch);
  P.part_val = reinterpret_cast<float *>(static_cast<unsigned char *>(scratch) + sizeof(hb::Ctrl));
  P.part_idx = reinterpret_cast<int *>(P.part_val + kNoAllocCtas * kNoAllocBatch);
  P.nslots = nslots;
  P.red_rows = red_rows;
  P.per_warp = per_warp;
  P.limit_ns = kDefaultLimitNs;
  return gemv_launch(dev, mb, w8, G, smem, P, s, "hb_gemv_noalloc");
}

}  // extern "C"

// ------------------------------------------------------------ sampling ------
struct hb_sampler {
  int device = 0;
  int vocab = 0;
  int rows = 1;              // rows selectable in one batch
  cudaStream_t own_stream = nullptr;
  float *d_in = nullptr, *d_s = nullptr, *d_e = nullptr;  // d_s, d_e: [rows][vocab]
  int2 *d_leaves = nullptr, *d_nodes = nullptr;
  int *d_levels = nullptr;
  int n_leaves = 0, n_nodes = 0, n_levels = 0;
  // [2 rows: out][rows x kMaxHistory: history tokens][rows x kMaxBias: bias tokens]
  int *d_ints = nullptr;
  // [rows x kMaxHistory: history counts][rows x kMaxBias: bias values]
  float *d_floats = nullptr;
  int *h_ints = nullptr;     // pinned staging, same layouts
  float *h_floats = nullptr;
  hb::SampleParams *d_params = nullptr, *h_params = nullptr;  // [rows]
  double *d_lp = nullptr, *h_lp = nullptr;  // [1 + kMaxTopLogprobs] log-probabilities
  int *d_lp_ids = nullptr, *h_lp_ids = nullptr;  // [kMaxTopLogprobs + 1]
  // the grid-wide kernel for single selections over large vocabularies
  int grid_ctas = 0;
  hb::SampleGrid grid{};
};

namespace {

constexpr int kMaxHistory = 8192;
constexpr int kMaxBias = 1024;  // MAX_LOGIT_BIAS_ENTRIES of the reference
constexpr int kGridMinVocab = 16384;  // below: one thread block selects

// NumPy's pairwise reduction tree of n values (np.add.reduce on a contiguous
// float array): leaves are runs of at most 128 values, a longer run splits
// at half its length rounded down to a multiple of 8.  Leaves are numbered
// left to right; internal nodes are then sorted by height so the device can
// combine one height per step.
struct PairwisePlan {
  std::vector<int2> leaves;
  std::vector<int2> nodes;
  std::vector<int> level_end;
};

void plan_rec(int lo, int n, std::vector<int2> &leaves, std::vector<int3> &internal, int &id, int &height) {
  if (n <= 128) {
    id = static_cast<int>(leaves.size());
    leaves.push_back(make_int2(lo, n));
    height = 0;
    return;
  }
  int n2 = n / 2;
  n2 -= n2 % 8;
  int lid, lh, rid, rh;
  plan_rec(lo, n2, leaves, internal, lid, lh);
  plan_rec(lo + n2, n - n2, leaves, internal, rid, rh);
  height = 1 + (lh > rh ? lh : rh);
  id = -1 - static_cast<int>(internal.size());  // provisional id of an internal node
  internal.push_back(make_int3(lid, rid, height));
}

PairwisePlan pairwise_plan(int n) {
  PairwisePlan pl;
  std::vector<int3> internal;
  int id = 0, h = 0;
  plan_rec(0, n, pl.leaves, internal, id, h);
  const int L = static_cast<int>(pl.leaves.size());
  std::vector<int> order(internal.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int>(i);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return internal[a].z < internal[b].z; });
  std::vector<int> final_id(internal.size());
  for (size_t k = 0; k < order.size(); ++k) final_id[order[k]] = L + static_cast<int>(k);
  auto resolve = [&](int v) { return v >= 0 ? v : final_id[-1 - v]; };
  int cur = 1;
  for (size_t k = 0; k < order.size(); ++k) {
    const int3 nd = internal[order[k]];
    if (nd.z != cur) {
      pl.level_end.push_back(static_cast<int>(k));
      cur = nd.z;
    }
    pl.nodes.push_back(make_int2(resolve(nd.x), resolve(nd.y)));
  }
  if (!order.empty()) pl.level_end.push_back(static_cast<int>(order.size()));
  return pl;
}

int sampler_fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_lib_error = buf;
  return code;
}

#define HB_SCUDA(call)                                                                 \
  do {                                                                                 \
    cudaError_t err_ = (call);                                                         \
    if (err_ != cudaSuccess) return sampler_fail(HB_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(err_)); \
  } while (0)

template <class T>
int sampler_alloc(T **p, size_t count) {
  HB_SCUDA(cudaMalloc(reinterpret_cast<void **>(p), sizeof(T) * (count ? count : 1)));
  return HB_OK;
}

// Validate one selection and stage its parameters for row `r` of the
// sampler's scratch (P points at device memory; the host lists sit in the
// pinned staging until sampler_upload).  The caller has made the sampler's
// device current.
int sampler_prepare(hb_sampler *sp, int r, const float *logits_dev, const hb_sampling *q, hb::SampleParams &P) {
  const int V = sp->vocab;
  if (!q) return sampler_fail(HB_ERR_INVALID_ARG, "params is NULL");
  auto finite = [](double v) { return v == v && v - v == 0.0; };
  if (!finite(q->temperature) || q->temperature < 0.f)
    return sampler_fail(HB_ERR_INVALID_ARG, "temperature must be finite and >= 0");
  if (!finite(q->top_p) || !(q->top_p > 0.f) || q->top_p > 1.f)
    return sampler_fail(HB_ERR_INVALID_ARG, "top_p must be in (0, 1]");
  if (q->top_k < 0) return sampler_fail(HB_ERR_INVALID_ARG, "top_k cannot be negative");
  if (!finite(q->repetition_penalty) || !(q->repetition_penalty > 0.f) || !finite(q->presence_penalty) ||
      !finite(q->frequency_penalty))
    return sampler_fail(HB_ERR_INVALID_ARG, "penalties must be finite (repetition > 0)");
  if (q->n_history < 0 || q->n_history > kMaxHistory || (q->n_history && (!q->history_tokens || !q->history_counts)))
    return sampler_fail(HB_ERR_INVALID_ARG, "history of %d tokens (at most %d)", q->n_history, kMaxHistory);
  if (q->n_bias < 0 || q->n_bias > kMaxBias || (q->n_bias && (!q->bias_tokens || !q->bias_values)))
    return sampler_fail(HB_ERR_INVALID_ARG, "logit bias of %d entries (at most %d)", q->n_bias, kMaxBias);
  for (int i = 0; i < q->n_history; ++i)
    if (q->history_tokens[i] < 0 || q->history_tokens[i] >= V)
      return sampler_fail(HB_ERR_INVALID_ARG, "history token %d outside the vocabulary", q->history_tokens[i]);
  for (int i = 0; i < q->n_bias; ++i)
    if (q->bias_tokens[i] < 0 || q->bias_tokens[i] >= V || !finite(q->bias_values[i]))
      return sampler_fail(HB_ERR_INVALID_ARG, "logit bias entry %d invalid", i);
  const bool neutral = q->repetition_penalty == 1.f && q->presence_penalty == 0.f && q->frequency_penalty == 0.f;
  // the reference's `greedy`: nothing can reorder the logits -> argmax, no draw
  const bool greedy = neutral && (q->temperature == 0.f || q->top_k == 1) && q->n_bias == 0;
  const bool draws = !greedy && q->temperature != 0.f;
  if (draws && !(q->uniform >= 0.0 && q->uniform < 1.0))
    return sampler_fail(HB_ERR_INVALID_ARG, "uniform must be in [0, 1)");
  const int R = sp->rows;
  P = hb::SampleParams{};
  P.logits = logits_dev;
  P.s = sp->d_s + static_cast<size_t>(r) * V;
  P.e = sp->d_e + static_cast<size_t>(r) * V;
  P.V = V;
  P.temperature = greedy ? 0.f : q->temperature;
  P.top_p = q->top_p;
  P.top_k = q->top_k;
  P.rep = q->repetition_penalty;
  P.pres = q->presence_penalty;
  P.freq = q->frequency_penalty;
  P.u = q->uniform;
  // penalties apply only when one of them is not neutral (sampling.py:341-346)
  P.n_hist = (greedy || neutral) ? 0 : q->n_history;
  P.n_bias = greedy ? 0 : q->n_bias;
  const size_t hist_off = static_cast<size_t>(r) * kMaxHistory, bias_off = static_cast<size_t>(r) * kMaxBias;
  int *h_htok = sp->h_ints + 2 * R + hist_off, *h_btok = sp->h_ints + 2 * R + static_cast<size_t>(R) * kMaxHistory + bias_off;
  float *h_hcnt = sp->h_floats + hist_off, *h_bval = sp->h_floats + static_cast<size_t>(R) * kMaxHistory + bias_off;
  for (int i = 0; i < P.n_hist; ++i) {
    h_htok[i] = q->history_tokens[i];
    h_hcnt[i] = q->history_counts[i];
  }
  for (int i = 0; i < P.n_bias; ++i) {
    h_btok[i] = q->bias_tokens[i];
    h_bval[i] = q->bias_values[i];
  }
  P.hist_tok = sp->d_ints + 2 * R + hist_off;
  P.bias_tok = sp->d_ints + 2 * R + static_cast<size_t>(R) * kMaxHistory + bias_off;
  P.hist_cnt = sp->d_floats + hist_off;
  P.bias_val = sp->d_floats + static_cast<size_t>(R) * kMaxHistory + bias_off;
  P.leaves = sp->d_leaves;
  P.n_leaves = sp->n_leaves;
  P.nodes = sp->d_nodes;
  P.n_nodes = sp->n_nodes;
  P.level_end = sp->d_levels;
  P.n_levels = sp->n_levels;
  P.out = sp->d_ints + 2 * r;
  return HB_OK;
}

// Copy a prepared row's lists from the staging to the device.
int sampler_upload(hb_sampler *sp, cudaStream_t stream, const hb::SampleParams &P) {
  const ptrdiff_t ti = P.hist_tok - sp->d_ints, bi = P.bias_tok - sp->d_ints;
  const ptrdiff_t tf = P.hist_cnt - sp->d_floats, bf = P.bias_val - sp->d_floats;
  if (P.n_hist) {
    HB_SCUDA(cudaMemcpyAsync(sp->d_ints + ti, sp->h_ints + ti, sizeof(int) * P.n_hist, cudaMemcpyHostToDevice, stream));
    HB_SCUDA(cudaMemcpyAsync(sp->d_floats + tf, sp->h_floats + tf, sizeof(float) * P.n_hist, cudaMemcpyHostToDevice, stream));
  }
  if (P.n_bias) {
    HB_SCUDA(cudaMemcpyAsync(sp->d_ints + bi, sp->h_ints + bi, sizeof(int) * P.n_bias, cudaMemcpyHostToDevice, stream));
    HB_SCUDA(cudaMemcpyAsync(sp->d_floats + bf, sp->h_floats + bf, sizeof(float) * P.n_bias, cudaMemcpyHostToDevice, stream));
  }
  return HB_OK;
}

// Select on `stream` from device logits.  The caller has made the sampler's
// device current.
int sampler_run(hb_sampler *sp, cudaStream_t stream, const float *logits_dev, const hb_sampling *q,
                int32_t *token_out) {
  if (!token_out) return sampler_fail(HB_ERR_INVALID_ARG, "token_out is NULL");
  hb::SampleParams P;
  int rc;
  if ((rc = sampler_prepare(sp, 0, logits_dev, q, P)) || (rc = sampler_upload(sp, stream, P))) return rc;
  if (sp->grid_ctas > 0) {
    void *args[] = {&P, &sp->grid};
    HB_SCUDA(cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(&hb::sample_grid_kernel), dim3(sp->grid_ctas),
                                         dim3(hb::kSampThreads), args, sizeof(hb::SampleSmem), stream));
  } else {
    hb::sample_kernel<<<1, hb::kSampThreads, sizeof(hb::SampleSmem), stream>>>(P);
  }
  HB_SCUDA(cudaGetLastError());
  HB_SCUDA(cudaMemcpyAsync(sp->h_ints, sp->d_ints, sizeof(int) * 2, cudaMemcpyDeviceToHost, stream));
  HB_SCUDA(cudaStreamSynchronize(stream));
  if (sp->h_ints[1] != 0) {
    *token_out = -1;
    return sampler_fail(HB_ERR_UNSUPPORTED, "top_p keeps more than %d candidates: select on the host", hb::kTopPMax);
  }
  *token_out = sp->h_ints[0];
  return HB_OK;
}

// Several selections in one launch: entry k from logits row rows[k] of
// `logits_dev` ([rows][vocab]); tokens_out[k] = -1 where the top-p nucleus
// is too large for the device.
int sampler_run_batch(hb_sampler *sp, cudaStream_t stream, const float *logits_dev, int n, const int32_t *rows,
                      const hb_sampling *q, int32_t *tokens_out, int max_row) {
  if (!rows || !q || !tokens_out) return sampler_fail(HB_ERR_INVALID_ARG, "rows, params or tokens_out is NULL");
  if (n < 1 || n > sp->rows) return sampler_fail(HB_ERR_INVALID_ARG, "%d selections outside [1, %d]", n, sp->rows);
  for (int k = 0; k < n; ++k) {
    if (rows[k] < 0 || rows[k] >= max_row) return sampler_fail(HB_ERR_INVALID_ARG, "row %d outside the batch", rows[k]);
    int rc = sampler_prepare(sp, k, logits_dev + static_cast<size_t>(rows[k]) * sp->vocab, q + k, sp->h_params[k]);
    if (!rc) rc = sampler_upload(sp, stream, sp->h_params[k]);
    if (rc) return rc;
  }
  HB_SCUDA(cudaMemcpyAsync(sp->d_params, sp->h_params, sizeof(hb::SampleParams) * n, cudaMemcpyHostToDevice, stream));
  hb::sample_batch_kernel<<<n, hb::kSampThreads, sizeof(hb::SampleSmem), stream>>>(sp->d_params);
  HB_SCUDA(cudaGetLastError());
  HB_SCUDA(cudaMemcpyAsync(sp->h_ints, sp->d_ints, sizeof(int) * 2 * n, cudaMemcpyDeviceToHost, stream));
  HB_SCUDA(cudaStreamSynchronize(stream));
  for (int k = 0; k < n; ++k) tokens_out[k] = sp->h_ints[2 * k + 1] != 0 ? -1 : sp->h_ints[2 * k];
  return HB_OK;
}

int sampler_logprobs_run(hb_sampler *sp, cudaStream_t stream, const float *logits_dev, int token, int n_top,
                         double *token_logprob, int32_t *top_ids, double *top_logprobs) {
  const int V = sp->vocab;
  if (!token_logprob || (n_top > 0 && (!top_ids || !top_logprobs)))
    return sampler_fail(HB_ERR_INVALID_ARG, "output pointer is NULL");
  if (token < 0 || token >= V) return sampler_fail(HB_ERR_INVALID_ARG, "token %d outside the vocabulary", token);
  if (n_top < 0 || n_top > hb::kMaxTopLogprobs || n_top > V)
    return sampler_fail(HB_ERR_INVALID_ARG, "top_logprobs %d outside [0, %d]", n_top, hb::kMaxTopLogprobs);
  hb::SampleParams P{};
  P.logits = logits_dev;
  P.s = sp->d_s;
  P.e = sp->d_e;
  P.V = V;
  P.leaves = sp->d_leaves;
  P.n_leaves = sp->n_leaves;
  P.nodes = sp->d_nodes;
  P.n_nodes = sp->n_nodes;
  P.level_end = sp->d_levels;
  P.n_levels = sp->n_levels;
  hb::logprob_kernel<<<1, hb::kSampThreads, sizeof(hb::SampleSmem), stream>>>(P, token, n_top, sp->d_lp, sp->d_lp_ids);
  HB_SCUDA(cudaGetLastError());
  HB_SCUDA(cudaMemcpyAsync(sp->h_lp, sp->d_lp, sizeof(double) * (1 + n_top), cudaMemcpyDeviceToHost, stream));
  HB_SCUDA(cudaMemcpyAsync(sp->h_lp_ids, sp->d_lp_ids, sizeof(int) * (n_top + 1), cudaMemcpyDeviceToHost, stream));
  HB_SCUDA(cudaStreamSynchronize(stream));
  if (sp->h_lp_ids[n_top] != 0) return sampler_fail(HB_ERR_INVALID_ARG, "logits contain no finite value");
  *token_logprob = sp->h_lp[0];
  for (int i = 0; i < n_top; ++i) {
    top_ids[i] = sp->h_lp_ids[i];
    top_logprobs[i] = sp->h_lp[1 + i];
  }
  return HB_OK;
}

}  // namespace

// A sampler with scratch for `rows` selections per launch (the engine's has
// one per batch row).
int sampler_create_rows(int vocab, int device, int rows, hb_sampler **out);

extern "C" {

int hb_sampler_create(int vocab, int device, hb_sampler **out) { return sampler_create_rows(vocab, device, 1, out); }

}  // extern "C"

int sampler_create_rows(int vocab, int device, int rows, hb_sampler **out) {
  if (!out) return sampler_fail(HB_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  if (vocab < 1 || vocab > hb::kSampMaxVocab)
    return sampler_fail(HB_ERR_UNSUPPORTED, "vocabulary of %d outside [1, %d]", vocab, hb::kSampMaxVocab);
  DeviceScope device_scope_(device);
  if (!device_scope_.ok) return sampler_fail(HB_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  hb_sampler *sp = new hb_sampler;
  sp->device = device;
  sp->vocab = vocab;
  sp->rows = rows;
  auto bail = [&](int rc) {
    hb_sampler_destroy(sp);
    return rc;
  };
  const PairwisePlan pl = pairwise_plan(vocab);
  sp->n_leaves = static_cast<int>(pl.leaves.size());
  sp->n_nodes = static_cast<int>(pl.nodes.size());
  sp->n_levels = static_cast<int>(pl.level_end.size());
  int rc;
  const size_t n_ints = static_cast<size_t>(rows) * (2 + kMaxHistory + kMaxBias);
  const size_t n_floats = static_cast<size_t>(rows) * (kMaxHistory + kMaxBias);
  if ((rc = sampler_alloc(&sp->d_in, vocab)) || (rc = sampler_alloc(&sp->d_s, static_cast<size_t>(rows) * vocab)) ||
      (rc = sampler_alloc(&sp->d_e, static_cast<size_t>(rows) * vocab)) || (rc = sampler_alloc(&sp->d_leaves, sp->n_leaves)) ||
      (rc = sampler_alloc(&sp->d_nodes, sp->n_nodes)) || (rc = sampler_alloc(&sp->d_levels, sp->n_levels)) ||
      (rc = sampler_alloc(&sp->d_ints, n_ints)) || (rc = sampler_alloc(&sp->d_floats, n_floats)) ||
      (rc = sampler_alloc(&sp->d_params, rows)) ||
      (rc = sampler_alloc(&sp->d_lp, 1 + hb::kMaxTopLogprobs)) ||
      (rc = sampler_alloc(&sp->d_lp_ids, hb::kMaxTopLogprobs + 1)))
    return bail(rc);
  if (cudaHostAlloc(reinterpret_cast<void **>(&sp->h_ints), sizeof(int) * n_ints, cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&sp->h_floats), sizeof(float) * n_floats, cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&sp->h_params), sizeof(hb::SampleParams) * rows, cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&sp->h_lp), sizeof(double) * (1 + hb::kMaxTopLogprobs),
                    cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&sp->h_lp_ids), sizeof(int) * (hb::kMaxTopLogprobs + 1),
                    cudaHostAllocDefault) != cudaSuccess)
    return bail(sampler_fail(HB_ERR_CUDA, "pinned host allocation failed"));
  if (cudaMemcpy(sp->d_leaves, pl.leaves.data(), sizeof(int2) * sp->n_leaves, cudaMemcpyHostToDevice) != cudaSuccess ||
      (sp->n_nodes && cudaMemcpy(sp->d_nodes, pl.nodes.data(), sizeof(int2) * sp->n_nodes, cudaMemcpyHostToDevice) != cudaSuccess) ||
      (sp->n_levels && cudaMemcpy(sp->d_levels, pl.level_end.data(), sizeof(int) * sp->n_levels, cudaMemcpyHostToDevice) != cudaSuccess))
    return bail(sampler_fail(HB_ERR_CUDA, "sampler plan upload failed"));
  if (cudaFuncSetAttribute(reinterpret_cast<const void *>(&hb::sample_kernel),
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(hb::SampleSmem))) != cudaSuccess ||
      cudaFuncSetAttribute(reinterpret_cast<const void *>(&hb::sample_batch_kernel),
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(hb::SampleSmem))) != cudaSuccess ||
      cudaFuncSetAttribute(reinterpret_cast<const void *>(&hb::logprob_kernel),
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(hb::SampleSmem))) != cudaSuccess ||
      cudaFuncSetAttribute(reinterpret_cast<const void *>(&hb::sample_grid_kernel),
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(hb::SampleSmem))) != cudaSuccess ||
      cudaStreamCreateWithFlags(&sp->own_stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(sampler_fail(HB_ERR_CUDA, "sampler set-up failed"));
  // single selections over a large vocabulary spread over every SM
  int coop = 0, sms = 0, per_sm = 0;
  if (vocab >= kGridMinVocab && cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) == cudaSuccess &&
      coop && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess &&
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reinterpret_cast<const void *>(&hb::sample_grid_kernel),
                                                    hb::kSampThreads, sizeof(hb::SampleSmem)) == cudaSuccess &&
      per_sm >= 1) {
    const int G = sms;
    hb::SampleGrid &g = sp->grid;
    if ((rc = sampler_alloc(&g.leaf32, sp->n_leaves)) || (rc = sampler_alloc(&g.leaf64, sp->n_leaves)) ||
        (rc = sampler_alloc(&g.cta_f, G)) || (rc = sampler_alloc(&g.cta_i, G)) || (rc = sampler_alloc(&g.cta_d, G)) ||
        (rc = sampler_alloc(&g.hist, 8 * 256)) || (rc = sampler_alloc(&g.cand, hb::kTopPMax)) ||
        (rc = sampler_alloc(&g.ctr, 4)) || (rc = sampler_alloc(&g.fs, 4)) || (rc = sampler_alloc(&g.ds, 2)))
      return bail(rc);
    sp->grid_ctas = G;
  }
  cudaGetLastError();
  *out = sp;
  return HB_OK;
}

extern "C" {

int hb_sampler_select(hb_sampler *sp, const float *logits, int logits_on_device, const hb_sampling *params,
                      int32_t *token_out) {
  if (!sp || !logits) return sampler_fail(HB_ERR_INVALID_ARG, "sampler or logits is NULL");
  DeviceScope device_scope_(sp->device);
  if (!device_scope_.ok) return sampler_fail(HB_ERR_CUDA, "cudaSetDevice(%d) failed", sp->device);
  const float *dev = logits;
  if (!logits_on_device) {
    HB_SCUDA(cudaMemcpyAsync(sp->d_in, logits, sizeof(float) * sp->vocab, cudaMemcpyHostToDevice, sp->own_stream));
    dev = sp->d_in;
  }
  return sampler_run(sp, sp->own_stream, dev, params, token_out);
}

int hb_sampler_logprobs(hb_sampler *sp, const float *logits, int logits_on_device, int token, int n_top,
                        double *token_logprob, int32_t *top_ids, double *top_logprobs) {
  if (!sp || !logits) return sampler_fail(HB_ERR_INVALID_ARG, "sampler or logits is NULL");
  DeviceScope device_scope_(sp->device);
  if (!device_scope_.ok) return sampler_fail(HB_ERR_CUDA, "cudaSetDevice(%d) failed", sp->device);
  const float *dev = logits;
  if (!logits_on_device) {
    HB_SCUDA(cudaMemcpyAsync(sp->d_in, logits, sizeof(float) * sp->vocab, cudaMemcpyHostToDevice, sp->own_stream));
    dev = sp->d_in;
  }
  return sampler_logprobs_run(sp, sp->own_stream, dev, token, n_top, token_logprob, top_ids, top_logprobs);
}

int hb_sampler_destroy(hb_sampler *sp) {
  if (!sp) return HB_OK;
  DeviceScope device_scope_(sp->device);
  if (sp->own_stream) cudaStreamSynchronize(sp->own_stream);
  const hb::SampleGrid &g = sp->grid;
  void *dev[] = {sp->d_in, sp->d_s, sp->d_e, sp->d_leaves, sp->d_nodes, sp->d_levels, sp->d_ints, sp->d_floats,
                 sp->d_lp, sp->d_lp_ids, sp->d_params, g.leaf32, g.leaf64, g.cta_f, g.cta_i, g.cta_d, g.hist,
                 g.cand, g.ctr, g.fs, g.ds};
  for (void *p : dev)
    if (p) cudaFree(p);
  void *host[] = {sp->h_ints, sp->h_floats, sp->h_lp, sp->h_lp_ids, sp->h_params};
  for (void *p : host)
    if (p) cudaFreeHost(p);
  if (sp->own_stream) cudaStreamDestroy(sp->own_stream);
  delete sp;
  return HB_OK;
}

int hb_sample(hb_engine *e, int row, const hb_sampling *params, int32_t *token_out) {
  int rc = check_engine(e);
  if (rc) return rc;
  if (row < 0 || row >= kMaxBatch || row >= e->desc.max_batch)
    return fail(e, HB_ERR_INVALID_ARG, "row %d outside the batch", row);
  if (!e->sampler && (rc = sampler_create_rows(e->desc.vocab, e->device, kMaxBatch, &e->sampler)))
    return fail(e, rc, "%s", g_lib_error.c_str());
  rc = sampler_run(e->sampler, e->stream, e->d_logits + static_cast<size_t>(row) * e->desc.vocab, params, token_out);
  if (rc) return fail(e, rc, "%s", g_lib_error.c_str());
  return HB_OK;
}

int hb_sample_batch(hb_engine *e, int n, const int32_t *rows, const hb_sampling *params, int32_t *tokens_out) {
  int rc = check_engine(e);
  if (rc) return rc;
  if (!e->sampler && (rc = sampler_create_rows(e->desc.vocab, e->device, kMaxBatch, &e->sampler)))
    return fail(e, rc, "%s", g_lib_error.c_str());
  rc = sampler_run_batch(e->sampler, e->stream, e->d_logits, n, rows, params, tokens_out, e->desc.max_batch);
  if (rc) return fail(e, rc, "%s", g_lib_error.c_str());
  return HB_OK;
}

int hb_logprobs(hb_engine *e, int row, int token, int n_top, double *token_logprob, int32_t *top_ids,
                double *top_logprobs) {
  int rc = check_engine(e);
  if (rc) return rc;
  if (row < 0 || row >= kMaxBatch || row >= e->desc.max_batch)
    return fail(e, HB_ERR_INVALID_ARG, "row %d outside the batch", row);
  if (!e->sampler && (rc = sampler_create_rows(e->desc.vocab, e->device, kMaxBatch, &e->sampler)))
    return fail(e, rc, "%s", g_lib_error.c_str());
  rc = sampler_logprobs_run(e->sampler, e->stream, e->d_logits + static_cast<size_t>(row) * e->desc.vocab, token,
                            n_top, token_logprob, top_ids, top_logprobs);
  if (rc) return fail(e, rc, "%s", g_lib_error.c_str());
  return HB_OK;
}

int hb_read_logits(hb_engine *e, int n_rows, float *logits_out) {
  int rc = check_engine(e);
  if (rc) return rc;
  if (!logits_out || n_rows < 1 || n_rows > e->desc.max_batch)
    return fail(e, HB_ERR_INVALID_ARG, "%d rows outside [1, %d] or NULL output", n_rows, e->desc.max_batch);
  HB_CUDA(e, cudaMemcpyAsync(logits_out, e->d_logits, sizeof(float) * e->desc.vocab * n_rows, cudaMemcpyDeviceToHost,
                             e->stream));
  HB_CUDA(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

}  // extern "C"

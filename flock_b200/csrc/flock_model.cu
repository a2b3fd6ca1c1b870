// Model: kernels/model.ts on B200.  ids -> embedding gather -> held layers ->
// output_norm -> tied (or untied) Q8_0 head -> argmax, everything on the
// device; the host sees one int32 per generated token.
//
// Device-side state makes a decode step replayable as one CUDA graph: the
// position lives in a {pos, n_last} control block that layer 0's first
// kernel advances, the head's last CTA writes the chosen id into ids[0]
// (the next step's embedding input) and into a per-position history, so a
// greedy decode loop needs no host round trip at all.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "decode_mk.cuh"
#include "flock_internal.h"
#include "stream_engine.h"
#include "gemv.cuh"
#include "ops.cuh"

using namespace flock;

struct flock_model {
  flock_dev* dev = nullptr;
  flock_layer_config cfg{};
  int vocab = 0, n_layers = 0, held = 0;
  std::vector<flock_layer*> layers;
  const flock_tensor* embd = nullptr;
  const flock_tensor* out_norm = nullptr;
  const flock_tensor* head = nullptr;  // lm-head: embd when tied
  Workspace ws;
  DBuf ctl, ids, hist, logits, normed, am_val, am_idx, am_count, am_best_val;
  int pos = 0;  // host mirror of ctl[0] after the last step
  // the kernel graph of one decode step, and of DECODE_GRAPH_TOKENS steps
  // in a row (device-fed decode runs: no graph boundary, so each step's
  // first launch overlaps the previous step's last one)
  cudaGraphExec_t decode_graph = nullptr, decode_graph_run = nullptr;
  // pinned host slots of a one-token step: [0] the id going in, [1] the id
  // coming back (both copies asynchronous on the model's stream)
  int32_t* h_io = nullptr;
  // persistent decode kernel
  int decode_mode = FLOCK_DECODE_KERNELS;
  bool mk_ok = false;       // shape fits the persistent kernel
  DBuf mk_layers, mk_bar, mk_err, mk_trace, mk_gemv, mk_attn;
  MkArgs mk{};
  size_t mk_smem = 0;
  int mk_grid = 0;
  // streaming persistent decode kernel (weights through shared-memory rings)
  StEngine st;
  // tensor parallel: this rank holds vocab rows [tp_start[r], tp_start[r+1])
  // of the head; layers exchange partials over `tp`
  flock_comm* tp = nullptr;
  PeerXchg* xchg = nullptr;   // fused peer exchange for decode steps (null: NCCL)
  int tp_exchange = FLOCK_TP_PEER;
  int tp_rank = 0, tp_n = 1, tp_chunk = 0;
  std::vector<int64_t> tp_start;
  DBuf tp_best, tp_bests, tp_logits;
};

namespace {

int enqueue_embed(flock_model* m, int n) {
  EmbedArgs a = {};
  a.qs = m->embd->qs.as<uint8_t>();
  a.sc = m->embd->sc.as<uint16_t>();
  a.ids = m->ids.as<int32_t>();
  a.out = m->ws.h.as<float>();
  a.n_tokens = n;
  a.hidden = m->cfg.hidden;
  a.sc_stride = m->embd->sc_stride;
  a.vocab = (int)m->embd->rows;
  if (m->held > 0) {
    const flock_tensor* q = m->layers[0]->w[W_Q];
    a.pf.ptr[0] = q->qs.as<uint8_t>();
    a.pf.bytes[0] = q->qs.bytes & ~(uint64_t)15;
    a.pf.n = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n < 64 ? 64 : n);
  cfg.blockDim = dim3(256);
  cfg.stream = m->dev->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FLOCK_CK(cudaLaunchKernelEx(&cfg, k_embed, a));
  return FLOCK_OK;
}

// Layers over ws.h ([n][hidden]); layer 0 advances the shared position.
// Each layer's host key count is set to the model's position first: a
// multi-token step sizes host-side work by it (the tensor-core attention's
// image of earlier keys), and the chunks of one prompt advance m->pos
// between calls.
int enqueue_layers(flock_model* m, int n) {
  for (int i = 0; i < m->held; i++) m->layers[i]->n_keys = m->pos;
  for (int i = 0; i < m->held; i++) {
    PrefetchList pf = {};
    if (i + 1 < m->held) {
      const flock_tensor* q = m->layers[i + 1]->w[W_Q];
      pf.ptr[0] = q->qs.as<uint8_t>();
      pf.bytes[0] = q->qs.bytes & ~(uint64_t)15;
      const flock_tensor* k = m->layers[i + 1]->w[W_K];
      pf.ptr[1] = k->qs.as<uint8_t>();
      pf.bytes[1] = k->qs.bytes & ~(uint64_t)15;
      const flock_tensor* v = m->layers[i + 1]->w[W_V];
      pf.ptr[2] = v->qs.as<uint8_t>();
      pf.bytes[2] = v->qs.bytes & ~(uint64_t)15;
      pf.n = 3;
    }
    m->ws.defer_down = i + 1 < m->held;
    const int rc = layer_enqueue(m->layers[i], n, i == 0, pf, true);
    m->ws.defer_down = false;
    if (rc) {
      m->ws.down_pending = 0;
      return rc;
    }
  }
  return FLOCK_OK;
}

// Tensor parallel: the ranks' (value, global index) maxima in rank order ->
// the token, by reduceShardArgmax's rule (shard_ref.ts:437; greater value,
// or equal value and lower index), into ids[0].
static __global__ void k_tp_argmax(const uint32_t* bests, int n_ranks, int32_t* ids) {
  if (threadIdx.x != 0) return;
  float bv = __uint_as_float(bests[0]);
  uint32_t bi = bests[1];
  for (int r = 1; r < n_ranks; r++) {
    const float v = __uint_as_float(bests[2 * r]);
    const uint32_t ix = bests[2 * r + 1];
    if (am_better(v, ix, bv, bi)) {
      bv = v;
      bi = ix;
    }
  }
  ids[0] = (int32_t)bi;
}

// output_norm + lm-head + argmax on row `row` of ws.h.  Tensor parallel: the
// head is this rank's vocab rows; its (value, index) maximum is all-gathered
// and reduced, so every rank ends with the same id.
int enqueue_head(flock_model* m, int row) {
  GemvArgs a = {};
  GemvSeg s;
  s.qs = m->head->qs.as<uint8_t>();
  s.sc = m->head->sc.as<uint16_t>();
  s.out = m->tp ? m->tp_logits.as<float>() + (size_t)m->tp_rank * m->tp_chunk
                : m->logits.as<float>();
  s.rows = (int)m->head->rows;
  s.sc_stride = m->head->sc_stride;
  s.out_stride = (int)m->head->rows;
  a.seg[0] = s;
  a.nseg = 1;
  a.K = m->cfg.hidden;
  a.n_tokens = 1;
  a.x = m->ws.h.as<float>() + (size_t)row * m->cfg.hidden;
  a.x_stride = m->cfg.hidden;
  a.norm_gain = m->out_norm->data.as<float>();
  a.eps = m->cfg.eps;
  a.am_val = m->am_val.as<float>();
  a.am_idx = m->am_idx.as<uint32_t>();
  a.am_count = m->am_count.as<uint32_t>();
  a.am_best_val = m->am_best_val.as<float>();
  a.am_best_idx = m->ids.as<int32_t>();
  auto go = [&] {
    return m->cfg.matvec == FLOCK_MATVEC_FAST ? launch_gemv_fast(m->dev, QT_Q8, EPI_ARGMAX, a, true)
                                              : launch_gemv(m->dev, QT_Q8, EPI_ARGMAX, a, true);
  };
  if (!m->tp) return go();
  a.am_row_offset = (int)m->tp_start[m->tp_rank];
  a.am_best_val = m->tp_best.as<float>();
  a.am_best_idx = m->tp_best.as<int32_t>() + 1;
  FLOCK_TRY(go());
  FLOCK_TRY(comm_allgather_dev(m->tp, m->tp_best.p, m->tp_bests.p, 8));
  k_tp_argmax<<<1, 32, 0, m->dev->stream>>>(m->tp_bests.as<uint32_t>(), m->tp_n,
                                            m->ids.as<int32_t>());
  FLOCK_CK(cudaGetLastError());
  return FLOCK_OK;
}

// Wait for the model's stream: bounded by the communicator's deadline (which
// aborts it) when the step holds collectives.
int sync_model(flock_model* m) {
  if (m->tp) return comm_wait(m->tp);
  FLOCK_CK(cudaStreamSynchronize(m->dev->stream));
  return FLOCK_OK;
}

// Copy ids[0] (the chosen token) into hist[pos_last] on the device.
static __global__ void k_record(const int32_t* ids, const int* ctl, int32_t* hist, int cap) {
  pdl_wait();
  const int p = ctl[0] + ctl[1] - 1;
  if (p >= 0 && p < cap) hist[p] = ids[0];
}

int enqueue_record(flock_model* m) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(1);
  cfg.stream = m->dev->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FLOCK_CK(cudaLaunchKernelEx(&cfg, k_record, (const int32_t*)m->ids.as<int32_t>(),
                              (const int*)m->ctl.as<int>(), m->hist.as<int32_t>(),
                              m->cfg.max_keys));
  return FLOCK_OK;
}

int check_room(flock_model* m, int n) {
  if (m->pos + n > m->cfg.max_keys) {
    set_error("sequence would exceed maxKeys %d at %d", m->cfg.max_keys, m->pos + n);
    return FLOCK_E_STATE;
  }
  return FLOCK_OK;
}

int upload_ids(flock_model* m, const int32_t* ids, int n) {
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= m->vocab) {
      set_error("token id %d out of range 0..%d", ids[i], m->vocab - 1);
      return FLOCK_E_ARG;
    }
  FLOCK_CK(cudaMemcpyAsync(m->ids.p, ids, (size_t)n * 4, cudaMemcpyHostToDevice, m->dev->stream));
  return FLOCK_OK;
}

// model.ts:235 encodeTokens: chunks of maxPrefill; leaves the last chunk's
// rows in ws.h.  Returns the size of the last chunk.
int encode_tokens(flock_model* m, const int32_t* ids, int n, int* last_chunk) {
  if (n < 1) {
    set_error("no tokens");
    return FLOCK_E_ARG;
  }
  FLOCK_TRY(check_room(m, n));
  for (int off = 0; off < n; off += m->cfg.max_prefill) {
    const int c = (n - off) < m->cfg.max_prefill ? (n - off) : m->cfg.max_prefill;
    FLOCK_TRY(upload_ids(m, ids + off, c));
    FLOCK_TRY(enqueue_embed(m, c));
    FLOCK_TRY(enqueue_layers(m, c));
    m->pos += c;
    *last_chunk = c;
  }
  return FLOCK_OK;
}

// The persistent decode kernel's tables and launch shape (once per model).
int mk_prepare(flock_model* m) {
  const flock_layer_config& c = m->cfg;
  m->mk_ok = false;
  if (c.attention != FLOCK_ATTN_FAST || !m->embd || !m->head || m->held < 1 || c.head_dim != 128 ||
      c.n_heads / c.n_kv_heads > 4 || c.hidden > 4096 || m->tp || c.matvec != FLOCK_MATVEC_EXACT)
    return FLOCK_OK;
  int dev = m->dev->ordinal, coop = 0, smem_optin = 0;
  FLOCK_CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  FLOCK_CK(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (!coop) return FLOCK_OK;
  const int grid = m->dev->sm_count;
  const int splits = attn_max_splits(grid, c.n_kv_heads, c.max_keys);  // = the kernel graph's
  if (splits != m->ws.attn_splits) return FLOCK_OK;
  MkArgs& a = m->mk;
  a = MkArgs{};
  const size_t smem = mk_smem_bytes(c.hidden, c.n_heads * c.head_dim, c.ffn) + 1024;  // + static
  if (smem > (size_t)smem_optin) return FLOCK_OK;
  if (m->embd->dtype != FLOCK_Q8_0 || m->head->dtype != FLOCK_Q8_0) return FLOCK_OK;
  for (int i = 0; i < m->held; i++)
    for (int t = 0; t < 7; t++)
      if (m->layers[i]->w[t]->dtype != FLOCK_Q8_0) return FLOCK_OK;
  std::vector<MkLayer> tab(m->held);
  for (int i = 0; i < m->held; i++) {
    flock_layer* L = m->layers[i];
    for (int t = 0; t < 7; t++) {
      tab[i].qs[t] = L->w[t]->qs.as<uint8_t>();
      tab[i].sc[t] = L->w[t]->sc.as<uint16_t>();
      tab[i].sc_stride[t] = L->w[t]->sc_stride;
    }
    tab[i].attn_norm = L->w[W_ATTN_NORM]->data.as<float>();
    tab[i].q_norm = L->w[W_Q_NORM]->data.as<float>();
    tab[i].k_norm = L->w[W_K_NORM]->data.as<float>();
    tab[i].ffn_norm = L->w[W_FFN_NORM]->data.as<float>();
    tab[i].kcache = L->kcache.p;
    tab[i].vcache = L->vcache.p;
  }
  FLOCK_TRY(m->mk_layers.alloc(tab.size() * sizeof(MkLayer)));
  FLOCK_CK(cudaMemcpy(m->mk_layers.p, tab.data(), tab.size() * sizeof(MkLayer),
                      cudaMemcpyHostToDevice));
  FLOCK_TRY(m->mk_bar.alloc(16));
  FLOCK_TRY(m->mk_err.alloc(16));
  FLOCK_CK(cudaMemset(m->mk_err.p, 0, 16));
  a.layers = m->mk_layers.as<MkLayer>();
  a.n_layers = m->held;
  a.H = c.hidden;
  a.nH = c.n_heads;
  a.nKV = c.n_kv_heads;
  a.hd = c.head_dim;
  a.kv_bytes = (int)kv_elem_bytes(c);
  a.F = c.ffn;
  a.vocab = m->vocab;
  a.eps = c.eps;
  a.neox = c.rope_pairing == FLOCK_ROPE_NEOX;
  a.inv_freq = m->layers[0]->inv_freq.as<float>();
  a.embd_qs = m->embd->qs.as<uint8_t>();
  a.embd_sc = m->embd->sc.as<uint16_t>();
  a.embd_sc_stride = m->embd->sc_stride;
  a.head_qs = m->head->qs.as<uint8_t>();
  a.head_sc = m->head->sc.as<uint16_t>();
  a.head_sc_stride = m->head->sc_stride;
  a.out_norm = m->out_norm->data.as<float>();
  a.h = m->ws.h.as<float>();
  a.q = m->ws.q.as<float>();
  a.k = m->ws.k.as<float>();
  a.v = m->ws.v.as<float>();
  a.attn = m->ws.attn.as<float>();
  a.act = m->ws.act.as<float>();
  a.logits = m->logits.as<float>();
  a.ids = m->ids.as<int32_t>();
  a.hist = m->hist.as<int32_t>();
  a.hist_cap = c.max_keys;
  a.attn_part = m->ws.attn_part.as<float>();
  a.attn_count = m->ws.attn_count.as<uint32_t>();
  a.splits = splits;
  a.am_val = m->am_val.as<float>();
  a.am_idx = m->am_idx.as<uint32_t>();
  a.am_count = m->am_count.as<uint32_t>();
  a.am_best_val = m->am_best_val.as<float>();
  a.ctl = m->ctl.as<int>();
  a.bar = m->mk_bar.as<unsigned>();
  a.err = m->mk_err.as<int>();
  // the last layer streams the head's first rows into L2 (it exceeds L2)
  a.head_prefetch = (int64_t)48 << 20;
  // per-phase arguments: what each phase's kernel-graph launch would get
  // (n = 1, no step-control advance, no prefetch list)
  {
    auto seg = [](const flock_tensor* t, float* out, int out_stride) {
      GemvSeg s;
      s.qs = t->qs.as<uint8_t>();
      s.sc = t->sc.as<uint16_t>();
      s.out = out;
      s.rows = (int)t->rows;
      s.sc_stride = t->sc_stride;
      s.out_stride = out_stride;
      return s;
    };
    Workspace& ws = m->ws;
    const int qw = c.n_heads * c.head_dim, kvw = c.n_kv_heads * c.head_dim;
    std::vector<GemvArgs> gv((size_t)4 * m->held + 1);
    std::vector<AttnFastArgs> at((size_t)m->held);
    for (int i = 0; i < m->held; i++) {
      flock_layer* L = m->layers[i];
      GemvArgs* g = &gv[(size_t)4 * i];
      g[0] = GemvArgs{};
      g[0].seg[0] = seg(L->w[W_Q], ws.q.as<float>(), qw);
      g[0].seg[1] = seg(L->w[W_K], ws.k.as<float>(), kvw);
      g[0].seg[2] = seg(L->w[W_V], ws.v.as<float>(), kvw);
      g[0].nseg = 3;
      g[0].K = c.hidden;
      g[0].n_tokens = 1;
      g[0].x = ws.h.as<float>();
      g[0].x_stride = c.hidden;
      g[0].norm_gain = L->w[W_ATTN_NORM]->data.as<float>();
      g[0].eps = c.eps;
      g[1] = GemvArgs{};
      g[1].seg[0] = seg(L->w[W_O], ws.h.as<float>(), c.hidden);
      g[1].nseg = 1;
      g[1].K = qw;
      g[1].n_tokens = 1;
      g[1].x = ws.attn.as<float>();
      g[1].x_stride = qw;
      g[1].res = ws.h.as<float>();
      g[1].res_stride = c.hidden;
      g[2] = GemvArgs{};
      g[2].seg[0] = seg(L->w[W_GATE], ws.act.as<float>(), c.ffn);
      g[2].seg[1] = seg(L->w[W_UP], ws.act.as<float>(), c.ffn);
      g[2].nseg = 2;
      g[2].K = c.hidden;
      g[2].n_tokens = 1;
      g[2].x = ws.h.as<float>();
      g[2].x_stride = c.hidden;
      g[2].norm_gain = L->w[W_FFN_NORM]->data.as<float>();
      g[2].eps = c.eps;
      g[3] = GemvArgs{};
      g[3].seg[0] = seg(L->w[W_DOWN], ws.h.as<float>(), c.hidden);
      g[3].nseg = 1;
      g[3].K = c.ffn;
      g[3].n_tokens = 1;
      g[3].x = ws.act.as<float>();
      g[3].x_stride = c.ffn;
      g[3].res = ws.h.as<float>();
      g[3].res_stride = c.hidden;
      AttnFastArgs& aa = at[(size_t)i];
      aa = AttnFastArgs{};
      aa.q = ws.q.as<float>();
      aa.k = ws.k.as<float>();
      aa.v = ws.v.as<float>();
      aa.q_norm = L->w[W_Q_NORM]->data.as<float>();
      aa.k_norm = L->w[W_K_NORM]->data.as<float>();
      aa.inv_freq = L->inv_freq.as<float>();
      aa.kcache = L->kcache.p;
      aa.vcache = L->vcache.p;
      aa.kv_bf16 = c.kv_dtype == FLOCK_KV_BF16;
      aa.kv_fp8 = c.kv_dtype == FLOCK_KV_FP8;
      aa.out = ws.attn.as<float>();
      aa.part = ws.attn_part.as<float>();
      aa.count = ws.attn_count.as<uint32_t>();
      aa.n_heads = c.n_heads;
      aa.n_kv_heads = c.n_kv_heads;
      aa.head_dim = c.head_dim;
      aa.splits = splits;
      aa.eps = c.eps;
      aa.neox = c.rope_pairing == FLOCK_ROPE_NEOX;
      aa.chunk_cap = (c.max_keys + splits - 1) / splits;
      aa.combine = 1;
      aa.rope_cs = ws.rope.as<float2>();
      aa.rope_rows = ws.rope_rows;
    }
    GemvArgs& hg = gv[(size_t)4 * m->held];
    hg = GemvArgs{};
    hg.seg[0] = seg(m->head, m->logits.as<float>(), (int)m->head->rows);
    hg.nseg = 1;
    hg.K = c.hidden;
    hg.n_tokens = 1;
    hg.x = ws.h.as<float>();
    hg.x_stride = c.hidden;
    hg.norm_gain = m->out_norm->data.as<float>();
    hg.eps = c.eps;
    hg.am_val = m->am_val.as<float>();
    hg.am_idx = m->am_idx.as<uint32_t>();
    hg.am_count = m->am_count.as<uint32_t>();
    hg.am_best_val = m->am_best_val.as<float>();
    hg.am_best_idx = m->ids.as<int32_t>();
    FLOCK_TRY(m->mk_gemv.alloc(gv.size() * sizeof(GemvArgs)));
    FLOCK_CK(cudaMemcpy(m->mk_gemv.p, gv.data(), gv.size() * sizeof(GemvArgs),
                        cudaMemcpyHostToDevice));
    FLOCK_TRY(m->mk_attn.alloc(at.size() * sizeof(AttnFastArgs)));
    FLOCK_CK(cudaMemcpy(m->mk_attn.p, at.data(), at.size() * sizeof(AttnFastArgs),
                        cudaMemcpyHostToDevice));
    a.gemv = m->mk_gemv.as<GemvArgs>();
    a.attn_args = m->mk_attn.as<AttnFastArgs>();
  }
  FLOCK_TRY(kernel_setup((const void*)k_decode_mk, (int)smem));
  int per_sm = 0;
  FLOCK_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_mk, MK_THREADS, smem));
  if (per_sm < 1) return FLOCK_OK;
  // every CTA must be resident (cooperative launch); two per SM when they fit,
  // as the graph's GEMVs run (the attention phase loops CTAs over its items)
  m->mk_smem = smem;
  m->mk_grid = (per_sm >= 2 ? 2 : 1) * grid;
  if (m->mk_grid > 4096) return FLOCK_OK;
  m->mk_ok = true;
  return FLOCK_OK;
}

// The streaming engine's description of this model (once per model).
int st_prepare(flock_model* m) {
  const flock_layer_config& c = m->cfg;
  if (c.attention != FLOCK_ATTN_FAST) {
    m->st.why = "needs fast (split-K) attention";
    return FLOCK_OK;
  }
  if (c.matvec != FLOCK_MATVEC_EXACT) {
    m->st.why = "its matvecs are the exact-order ones (FLOCK_MATVEC_EXACT)";
    return FLOCK_OK;
  }
  if (c.kv_dtype == FLOCK_KV_FP8) {
    m->st.why = "its attention reads f32 or bf16 caches";
    return FLOCK_OK;
  }
  if (m->tp || !m->embd || !m->head || m->held < 1 || m->held != m->n_layers) {
    m->st.why = "needs a whole single-GPU model with its embedding and head";
    return FLOCK_OK;
  }
  StModelDesc d;
  d.H = c.hidden;
  d.nH = c.n_heads;
  d.nKV = c.n_kv_heads;
  d.hd = c.head_dim;
  d.F = c.ffn;
  d.vocab = m->vocab;
  d.n_layers = m->held;
  d.eps = c.eps;
  d.neox = c.rope_pairing == FLOCK_ROPE_NEOX;
  d.kv_bf16 = c.kv_dtype == FLOCK_KV_BF16;
  for (int i = 0; i < m->held; i++) {
    flock_layer* L = m->layers[i];
    for (int t = 0; t < W_COUNT; t++) d.w.push_back(L->w[t]);
    d.kcache.push_back(L->kcache.p);
    d.vcache.push_back(L->vcache.p);
  }
  d.embd = m->embd;
  d.head = m->head;
  d.out_norm = m->out_norm;
  d.inv_freq = m->layers[0]->inv_freq.as<float>();
  d.h_out = m->ws.h.as<float>();
  d.logits = m->logits.as<float>();
  d.ids = m->ids.as<int32_t>();
  d.hist = m->hist.as<int32_t>();
  d.hist_cap = c.max_keys;
  d.max_keys = c.max_keys;
  d.ctl = m->ctl.as<int>();
  return stream_prepare(m->dev, d, &m->st);
}

int enqueue_mk(flock_model* m) {
  FLOCK_CK(cudaMemsetAsync(m->mk_bar.p, 0, 4, m->dev->stream));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->mk_grid);
  cfg.blockDim = dim3(MK_THREADS);
  cfg.dynamicSmemBytes = m->mk_smem;
  cfg.stream = m->dev->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FLOCK_CK(cudaLaunchKernelEx(&cfg, k_decode_mk, m->mk));
  return FLOCK_OK;
}

// The device error words of the persistent kernel and the tensor-core
// prefill GEMMs; call after a synchronisation.
int check_device_errors(flock_model* m) {
  FLOCK_TRY(ws_check_errors(&m->ws));
  FLOCK_TRY(peer_xchg_check(m->xchg));
  if (m->decode_mode == FLOCK_DECODE_STREAM) return stream_check(&m->st);
  if (!m->mk_ok || m->decode_mode != FLOCK_DECODE_PERSISTENT) return FLOCK_OK;
  int err = 0;
  FLOCK_CK(cudaMemcpy(&err, m->mk_err.p, 4, cudaMemcpyDeviceToHost));
  if (err) {
    set_error("persistent decode kernel gave up waiting (%s timeout)",
              err == 2 ? "grid barrier" : "weight stream");
    cudaMemset(m->mk_err.p, 0, 4);
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

constexpr int DECODE_GRAPH_TOKENS = 8;

// Captures `tokens` decode steps (embed -> layers -> head -> record each)
// into one executable graph.
int capture_decode_steps(flock_model* m, int tokens, cudaGraphExec_t* out) {
  if (*out) return FLOCK_OK;
  cudaStream_t st = m->dev->stream;
  cudaGraph_t g = nullptr;
  FLOCK_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  int rc = FLOCK_OK;
  for (int i = 0; i < tokens && !rc; i++) {
    rc = enqueue_embed(m, 1);
    if (!rc) rc = enqueue_layers(m, 1);
    if (!rc) rc = enqueue_head(m, 0);
    if (!rc) rc = enqueue_record(m);
  }
  cudaError_t e = cudaStreamEndCapture(st, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) {
    set_error("decode graph capture failed: %s", cudaGetErrorString(e));
    return FLOCK_E_CUDA;
  }
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    *out = nullptr;
    set_error("decode graph instantiate failed: %s", cudaGetErrorString(e));
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

int capture_decode(flock_model* m) { return capture_decode_steps(m, 1, &m->decode_graph); }

// Drops the captured decode graphs (after the stream drains): the launches
// they hold change with the decode mode or the tensor-parallel exchange.
void drop_decode_graphs(flock_model* m) {
  if (!m->decode_graph && !m->decode_graph_run) return;
  cudaStreamSynchronize(m->dev->stream);
  if (m->decode_graph) cudaGraphExecDestroy(m->decode_graph);
  if (m->decode_graph_run) cudaGraphExecDestroy(m->decode_graph_run);
  m->decode_graph = m->decode_graph_run = nullptr;
}

// One single-token decode step on the stream: the persistent kernel (a
// barrier reset plus one cooperative launch; no graph, so profilers see the
// kernel) or the captured kernel graph.
int launch_decode(flock_model* m) {
  if (m->decode_mode == FLOCK_DECODE_STREAM && m->st.ok) {
    // the layers in one streaming launch, then the graph's head GEMV (its
    // 296-CTA register-pipelined stream beats the persistent grid's 148 CTAs
    // on the 165 MB head) with the fused argmax, and the history record
    FLOCK_TRY(stream_launch(&m->st, m->dev->stream));
    FLOCK_TRY(enqueue_head(m, 0));
    return enqueue_record(m);
  }
  if (m->decode_mode == FLOCK_DECODE_PERSISTENT && m->mk_ok) return enqueue_mk(m);
  if (m->decode_mode == FLOCK_DECODE_EAGER) {
    FLOCK_TRY(enqueue_embed(m, 1));
    FLOCK_TRY(enqueue_layers(m, 1));
    FLOCK_TRY(enqueue_head(m, 0));
    return enqueue_record(m);
  }
  FLOCK_TRY(capture_decode(m));
  FLOCK_CK(cudaGraphLaunch(m->decode_graph, m->dev->stream));
  return FLOCK_OK;
}

// n device-fed decode steps: the kernel graph of a one-GPU model runs them
// DECODE_GRAPH_TOKENS to a graph launch (the same kernels in the same order
// as n single-step launches); the other engines, and tensor-parallel ranks
// (whose graphs hold collectives), one step at a time.
int launch_decode_run(flock_model* m, int n) {
  const bool graph = !m->tp && !(m->decode_mode == FLOCK_DECODE_STREAM && m->st.ok) &&
                     !(m->decode_mode == FLOCK_DECODE_PERSISTENT && m->mk_ok) &&
                     m->decode_mode != FLOCK_DECODE_EAGER;
  int i = 0;
  if (graph && n >= DECODE_GRAPH_TOKENS) {
    FLOCK_TRY(capture_decode_steps(m, DECODE_GRAPH_TOKENS, &m->decode_graph_run));
    for (; i + DECODE_GRAPH_TOKENS <= n; i += DECODE_GRAPH_TOKENS)
      FLOCK_CK(cudaGraphLaunch(m->decode_graph_run, m->dev->stream));
  }
  for (; i < n; i++) FLOCK_TRY(launch_decode(m));
  return FLOCK_OK;
}

int need_head(flock_model* m) {
  if (!m->embd || !m->head) {
    set_error("this model holds no embedding/head (a layer-range stage)");
    return FLOCK_E_STATE;
  }
  return FLOCK_OK;
}

// Model.create body; tp != nullptr builds one rank of the tensor-parallel
// model (cfg is the rank's slice, `output` its vocab rows of the head).
int model_build(flock_dev* dev, const flock_layer_config* cfg, int vocab, int n_layers,
                flock_tensor* const* lt, const flock_tensor* embd, const flock_tensor* output_norm,
                const flock_tensor* output, int cut, flock_comm* tp, flock_model** out) {
  if (!dev || !cfg || !out || n_layers < 0 || (n_layers > 0 && !lt)) return FLOCK_E_ARG;
  if (cut < 0) cut = n_layers;
  if (cut > n_layers) {
    set_error("cut %d is not in 0..%d", cut, n_layers);
    return FLOCK_E_ARG;
  }
  if (embd && (embd->cols != cfg->hidden || embd->dtype != FLOCK_Q8_0)) {
    set_error("token_embd cols %lld != hidden %d", (long long)embd->cols, cfg->hidden);
    return FLOCK_E_ARG;
  }
  if (embd && (!output_norm || output_norm->dtype != FLOCK_F32 || output_norm->cols != cfg->hidden)) {
    set_error("output_norm.weight missing or not %d f32", cfg->hidden);
    return FLOCK_E_MISSING;
  }
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  flock_model* m = new flock_model();
  m->dev = dev_retain(dev);
  m->cfg = *cfg;
  m->vocab = vocab;
  m->n_layers = n_layers;
  m->embd = embd;
  m->out_norm = output_norm;
  m->head = output ? output : embd;
  int rc = FLOCK_OK;
  auto fail = [&](int r) {
    flock_model_free(m);
    return r;
  };
  int64_t head_rows = vocab;
  if (tp) {
    m->tp = tp;
    if ((rc = comm_rank(tp, &m->tp_rank, &m->tp_n))) return fail(rc);
    // the head's vocab rows per rank: shard_ref.ts:97 shardRanges(vocab, n, 1)
    const int64_t base = vocab / m->tp_n, extra = vocab % m->tp_n;
    m->tp_start.assign(m->tp_n + 1, 0);
    for (int r = 0; r < m->tp_n; r++) m->tp_start[r + 1] = m->tp_start[r] + base + (r < extra);
    m->tp_chunk = (int)(base + (extra > 0));
    head_rows = m->tp_start[m->tp_rank + 1] - m->tp_start[m->tp_rank];
    if ((rc = m->tp_best.alloc(16)) || (rc = m->tp_bests.alloc((size_t)m->tp_n * 8)) ||
        (rc = m->tp_logits.alloc((size_t)m->tp_n * m->tp_chunk * 4)))
      return fail(rc);
  }
  if ((rc = m->ws.alloc(*cfg, dev->sm_count, tp ? m->tp_n : 0))) return fail(rc);
  if ((rc = m->ctl.alloc(16))) return fail(rc);
  if (cudaMemset(m->ctl.p, 0, 16) != cudaSuccess) return fail(FLOCK_E_CUDA);
  if ((rc = m->ids.alloc((size_t)m->ws.P * 4 + 16))) return fail(rc);
  if ((rc = m->hist.alloc((size_t)cfg->max_keys * 4))) return fail(rc);
  if ((rc = m->logits.alloc((size_t)(vocab > 0 ? vocab : 1) * 4))) return fail(rc);
  if ((rc = m->normed.alloc((size_t)cfg->hidden * 4))) return fail(rc);
  if ((rc = m->am_val.alloc(4096 * 4)) || (rc = m->am_idx.alloc(4096 * 4)) ||
      (rc = m->am_count.alloc(16)) || (rc = m->am_best_val.alloc(16)))
    return fail(rc);
  if (cudaMemset(m->am_count.p, 0, 16) != cudaSuccess) return fail(FLOCK_E_CUDA);
  if (cudaHostAlloc((void**)&m->h_io, 16, cudaHostAllocDefault) != cudaSuccess) {
    m->h_io = nullptr;
    set_error("pinned host slot for the step ids could not be allocated");
    return fail(FLOCK_E_CUDA);
  }
  if (m->head && (m->head->cols != cfg->hidden || m->head->rows != head_rows)) {
    set_error("lm-head%s is %lldx%lld, want %lldx%d", tp ? " slice" : "",
              (long long)m->head->rows, (long long)m->head->cols, (long long)head_rows,
              cfg->hidden);
    return fail(FLOCK_E_ARG);
  }
  for (int i = 0; i < cut; i++) {
    const char* names[W_COUNT];
    flock_tensor* ts[W_COUNT];
    for (int s = 0; s < W_COUNT; s++) {
      names[s] = kTensorNames[s];
      ts[s] = lt[(size_t)i * W_COUNT + s];
    }
    flock_layer* L = nullptr;
    // all held layers share the model's workspace and position block
    if ((rc = layer_build(dev, cfg, W_COUNT, names, ts, &m->ws, m->ctl.as<int>(), &L)))
      return fail(rc);
    L->tp = tp;
    L->tp_n = m->tp_n;
    m->layers.push_back(L);
  }
  m->held = cut;
  if (tp) {
    // decode exchanges through peer memory when every rank maps every peer;
    // otherwise (the ranks agree) they stay on NCCL
    if (cfg->hidden > 16 * 1024 || peer_xchg_init(tp, cfg->hidden, &m->xchg) != FLOCK_OK)
      m->xchg = nullptr;
    for (auto* L : m->layers) L->xchg = m->xchg;
  }
  if ((rc = mk_prepare(m))) return fail(rc);
  if ((rc = st_prepare(m))) return fail(rc);
  *out = m;
  return FLOCK_OK;
}

}  // namespace

extern "C" {

int flock_model_create(flock_dev* dev, const flock_layer_config* cfg, int vocab, int n_layers,
                       flock_tensor* const* lt, const flock_tensor* embd,
                       const flock_tensor* output_norm, const flock_tensor* output, int cut,
                       flock_model** out) {
  return model_build(dev, cfg, vocab, n_layers, lt, embd, output_norm, output, cut, nullptr, out);
}

int flock_model_create_tp(flock_dev* dev, const flock_layer_config* cfg, int vocab, int n_layers,
                          flock_tensor* const* lt, const flock_tensor* embd,
                          const flock_tensor* output_norm, const flock_tensor* output_slice,
                          flock_comm* comm, flock_model** out) {
  if (!comm || !dev || !cfg) return FLOCK_E_ARG;
  int rank = 0, n = 1;
  FLOCK_TRY(comm_rank(comm, &rank, &n));
  if (comm_device(comm) != dev) {
    set_error("the communicator belongs to another device");
    return FLOCK_E_ARG;
  }
  if (!embd || !output_norm || !output_slice) {
    set_error("a tensor-parallel rank holds the embedding, output_norm and its head slice");
    return FLOCK_E_MISSING;
  }
  if (vocab < n) {
    set_error("vocab %d cannot be cut into %d head slices", vocab, n);
    return FLOCK_E_ARG;
  }
  return model_build(dev, cfg, vocab, n_layers, lt, embd, output_norm, output_slice, -1, comm,
                     out);
}

int flock_model_set_decode_mode(flock_model* m, int mode) {
  if (!m || (mode != FLOCK_DECODE_KERNELS && mode != FLOCK_DECODE_PERSISTENT &&
             mode != FLOCK_DECODE_EAGER && mode != FLOCK_DECODE_STREAM))
    return FLOCK_E_ARG;
  if (mode != m->decode_mode) drop_decode_graphs(m);
  m->decode_mode = mode;
  return FLOCK_OK;
}

int flock_model_trace(flock_model* m, int enable) {
  if (!m) return FLOCK_E_ARG;
  if (m->decode_mode == FLOCK_DECODE_STREAM && m->st.ok) return stream_trace(&m->st, enable != 0);
  if (!m->mk_ok) {
    set_error("phase tracing needs the persistent decode kernel, which this model cannot run");
    return FLOCK_E_UNSUPPORTED;
  }
  if (enable && !m->mk_trace.p) {
    const size_t n = (size_t)m->mk_grid * mk_trace_stride(m->held);
    FLOCK_TRY(m->mk_trace.alloc(n * 8));
    FLOCK_CK(cudaMemset(m->mk_trace.p, 0, n * 8));
  }
  m->mk.trace = enable ? m->mk_trace.as<unsigned long long>() : nullptr;
  return FLOCK_OK;
}

int flock_model_trace_read(flock_model* m, uint64_t* out, int64_t cap, int* n_ctas, int* stride) {
  if (!m || !n_ctas || !stride) return FLOCK_E_ARG;
  if (m->decode_mode == FLOCK_DECODE_STREAM && m->st.ok) {
    *n_ctas = m->st.grid;
    *stride = stream_trace_stride(&m->st);
    const int64_t n = (int64_t)*n_ctas * *stride;
    if (!m->st.trace.p) return FLOCK_E_STATE;
    if (!out || cap < n) return FLOCK_E_LIMIT;
    FLOCK_TRY(sync_model(m));
    FLOCK_CK(cudaMemcpy(out, m->st.trace.p, (size_t)n * 8, cudaMemcpyDeviceToHost));
    return FLOCK_OK;
  }
  *n_ctas = m->mk_grid;
  *stride = mk_trace_stride(m->held);
  const int64_t n = (int64_t)m->mk_grid * *stride;
  if (!m->mk_trace.p) return FLOCK_E_STATE;
  if (!out || cap < n) return FLOCK_E_LIMIT;
  FLOCK_TRY(sync_model(m));
  FLOCK_CK(cudaMemcpy(out, m->mk_trace.p, (size_t)n * 8, cudaMemcpyDeviceToHost));
  return FLOCK_OK;
}

int flock_model_set_tp_exchange(flock_model* m, int mode) {
  if (!m || (mode != FLOCK_TP_NCCL && mode != FLOCK_TP_PEER)) return FLOCK_E_ARG;
  if (!m->tp) {
    set_error("not a tensor-parallel model");
    return FLOCK_E_STATE;
  }
  if (mode == FLOCK_TP_PEER && !m->xchg) {
    set_error("the ranks could not map each other's memory; decode exchanges stay on NCCL");
    return FLOCK_E_UNSUPPORTED;
  }
  drop_decode_graphs(m);
  m->tp_exchange = mode;
  for (auto* L : m->layers) L->xchg = mode == FLOCK_TP_PEER ? m->xchg : nullptr;
  return FLOCK_OK;
}

int flock_model_get_tp_exchange(const flock_model* m, int* mode) {
  if (!m || !mode) return FLOCK_E_ARG;
  *mode = (m->tp && m->xchg && m->tp_exchange == FLOCK_TP_PEER) ? FLOCK_TP_PEER : FLOCK_TP_NCCL;
  return FLOCK_OK;
}

int flock_model_get_decode_mode(const flock_model* m, int* mode) {
  if (!m || !mode) return FLOCK_E_ARG;
  *mode = ((m->decode_mode == FLOCK_DECODE_PERSISTENT && !m->mk_ok) ||
           (m->decode_mode == FLOCK_DECODE_STREAM && !m->st.ok))
              ? FLOCK_DECODE_KERNELS
              : m->decode_mode;
  return FLOCK_OK;
}

int flock_model_free(flock_model* m) {
  if (!m) return FLOCK_OK;
  flock_dev* d = m->dev;
  cudaSetDevice(d->ordinal);
  cudaStreamSynchronize(d->stream);
  if (m->decode_graph) cudaGraphExecDestroy(m->decode_graph);
  if (m->decode_graph_run) cudaGraphExecDestroy(m->decode_graph_run);
  if (m->h_io) cudaFreeHost(m->h_io);
  for (auto* L : m->layers) flock_layer_free(L);
  peer_xchg_free(m->xchg);  // a collective: every rank frees its model
  delete m;
  dev_release(d);
  return FLOCK_OK;
}

int flock_model_reset(flock_model* m) { return flock_model_rewind(m, 0); }

int flock_model_rewind(flock_model* m, int n_keys) {
  if (!m || n_keys < 0 || n_keys > m->cfg.max_keys) return FLOCK_E_ARG;
  int ctl[4] = {n_keys, 0, 0, 0};
  FLOCK_CK(cudaMemcpyAsync(m->ctl.p, ctl, sizeof ctl, cudaMemcpyHostToDevice, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  m->pos = n_keys;
  for (auto* L : m->layers) L->n_keys = n_keys;
  return FLOCK_OK;
}

int flock_model_pos(const flock_model* m, int* out) {
  *out = m->pos;
  return FLOCK_OK;
}

int flock_model_held(const flock_model* m, int* out) {
  *out = m->held;
  return FLOCK_OK;
}

int flock_model_step(flock_model* m, const int32_t* ids, int n, int32_t* next_id) {
  if (!m || !ids || !next_id) return FLOCK_E_ARG;
  FLOCK_TRY(need_head(m));
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  if (n == 1 && m->held > 0) {
    // one decode step: the id goes up and the next comes back through the
    // pinned slots (the previous step's copies completed before it returned)
    FLOCK_TRY(check_room(m, 1));
    if (ids[0] < 0 || ids[0] >= m->vocab) {
      set_error("token id %d out of range 0..%d", ids[0], m->vocab - 1);
      return FLOCK_E_ARG;
    }
    m->h_io[0] = ids[0];
    FLOCK_CK(cudaMemcpyAsync(m->ids.p, m->h_io, 4, cudaMemcpyHostToDevice, m->dev->stream));
    FLOCK_TRY(launch_decode(m));
    m->pos += 1;
    for (auto* L : m->layers) L->n_keys = m->pos;
    FLOCK_CK(cudaMemcpyAsync(m->h_io + 1, m->ids.p, 4, cudaMemcpyDeviceToHost, m->dev->stream));
    FLOCK_TRY(sync_model(m));
    *next_id = m->h_io[1];
    return check_device_errors(m);
  }
  int last = 0;
  FLOCK_TRY(encode_tokens(m, ids, n, &last));
  FLOCK_TRY(enqueue_head(m, last - 1));
  FLOCK_TRY(enqueue_record(m));
  for (auto* L : m->layers) L->n_keys = m->pos;
  FLOCK_CK(cudaMemcpyAsync(next_id, m->ids.p, 4, cudaMemcpyDeviceToHost, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_decode_device(flock_model* m, int n_steps, int32_t* out_ids) {
  if (!m || n_steps < 0 || (n_steps > 0 && !out_ids)) return FLOCK_E_ARG;
  FLOCK_TRY(need_head(m));
  if (m->held == 0) return FLOCK_E_STATE;
  FLOCK_TRY(check_room(m, n_steps));
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  const int start = m->pos;
  FLOCK_TRY(launch_decode_run(m, n_steps));
  m->pos += n_steps;
  for (auto* L : m->layers) L->n_keys = m->pos;
  if (n_steps)
    FLOCK_CK(cudaMemcpyAsync(out_ids, m->hist.as<int32_t>() + start, (size_t)n_steps * 4,
                             cudaMemcpyDeviceToHost, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_generate(flock_model* m, const int32_t* prompt, int n_prompt, int max_tokens,
                         const int32_t* eos, int n_eos, int32_t* out_ids, int* n_out) {
  if (!m || !prompt || n_prompt < 1 || max_tokens < 0 || !n_out) return FLOCK_E_ARG;
  *n_out = 0;
  int32_t next = 0;
  FLOCK_TRY(flock_model_step(m, prompt, n_prompt, &next));
  for (int i = 0; i < max_tokens; i++) {
    bool stop = false;
    for (int e = 0; e < n_eos; e++) stop |= (eos[e] == next);
    if (stop) break;
    out_ids[(*n_out)++] = next;
    if (*n_out >= max_tokens) break;
    FLOCK_TRY(flock_model_step(m, &next, 1, &next));
  }
  return FLOCK_OK;
}

int flock_model_logits(flock_model* m, const int32_t* ids, int n, float* logits) {
  int32_t tok;
  FLOCK_TRY(flock_model_step(m, ids, n, &tok));
  if (!m->tp) {
    FLOCK_CK(cudaMemcpy(logits, m->logits.p, (size_t)m->vocab * 4, cudaMemcpyDeviceToHost));
    return FLOCK_OK;
  }
  // tensor parallel: gather the ranks' slices (in place, one padded slot per
  // rank) and lay them out contiguously; a collective like the step itself
  float* slots = m->tp_logits.as<float>();
  FLOCK_TRY(comm_allgather_dev(m->tp, slots + (size_t)m->tp_rank * m->tp_chunk, slots,
                               (size_t)m->tp_chunk * 4));
  for (int r = 0; r < m->tp_n; r++)
    FLOCK_CK(cudaMemcpyAsync(logits + m->tp_start[r], slots + (size_t)r * m->tp_chunk,
                             (size_t)(m->tp_start[r + 1] - m->tp_start[r]) * 4,
                             cudaMemcpyDeviceToHost, m->dev->stream));
  return sync_model(m);
}

int flock_model_hidden_state(flock_model* m, const int32_t* ids, int n, float* out) {
  if (!m || !ids || !out) return FLOCK_E_ARG;
  if (!m->embd) return need_head(m);
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  int last = 0;
  FLOCK_TRY(encode_tokens(m, ids, n, &last));
  for (auto* L : m->layers) L->n_keys = m->pos;
  FLOCK_CK(cudaMemcpyAsync(out, m->ws.h.as<float>() + (size_t)(last - 1) * m->cfg.hidden,
                           (size_t)m->cfg.hidden * 4, cudaMemcpyDeviceToHost, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_normed_state(flock_model* m, const int32_t* ids, int n, float* out) {
  if (!m || !ids || !out) return FLOCK_E_ARG;
  FLOCK_TRY(need_head(m));
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  int last = 0;
  FLOCK_TRY(encode_tokens(m, ids, n, &last));
  for (auto* L : m->layers) L->n_keys = m->pos;
  k_rmsnorm<<<1, 128, 0, m->dev->stream>>>(
      m->ws.h.as<float>() + (size_t)(last - 1) * m->cfg.hidden, m->out_norm->data.as<float>(),
      m->normed.as<float>(), m->cfg.hidden, 1, m->cfg.eps);
  FLOCK_CK(cudaGetLastError());
  FLOCK_TRY(enqueue_head(m, last - 1));
  FLOCK_CK(cudaMemcpyAsync(out, m->normed.p, (size_t)m->cfg.hidden * 4, cudaMemcpyDeviceToHost,
                           m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_embed(flock_model* m, const int32_t* ids, int n, float* out) {
  if (!m || !ids || !out || n < 1 || n > m->ws.P) return FLOCK_E_ARG;
  FLOCK_TRY(need_head(m));
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  FLOCK_TRY(upload_ids(m, ids, n));
  FLOCK_TRY(enqueue_embed(m, n));
  FLOCK_CK(cudaMemcpyAsync(out, m->ws.h.p, (size_t)n * m->cfg.hidden * 4, cudaMemcpyDeviceToHost,
                           m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_encode_partial(flock_model* m, const int32_t* ids, int n, int offset, float* out) {
  if (!m || !ids || !out) return FLOCK_E_ARG;
  if (offset >= 0 && offset != m->pos) {
    set_error("offset %d does not match this cache's position %d", offset, m->pos);
    return FLOCK_E_STATE;
  }
  if (n > m->cfg.max_prefill) {
    set_error("a lap of %d tokens exceeds maxPrefill %d", n, m->cfg.max_prefill);
    return FLOCK_E_STATE;
  }
  if (!m->embd) return need_head(m);
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  int last = 0;
  FLOCK_TRY(encode_tokens(m, ids, n, &last));
  for (auto* L : m->layers) L->n_keys = m->pos;
  FLOCK_CK(cudaMemcpyAsync(out, m->ws.h.p, (size_t)n * m->cfg.hidden * 4, cudaMemcpyDeviceToHost,
                           m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_project_hidden(flock_model* m, const float* flat, int seq, int32_t* next_id) {
  if (!m || !flat || seq < 1 || !next_id) return FLOCK_E_ARG;
  FLOCK_TRY(need_head(m));
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  FLOCK_CK(cudaMemcpyAsync(m->ws.h.p, flat + (size_t)(seq - 1) * m->cfg.hidden,
                           (size_t)m->cfg.hidden * 4, cudaMemcpyHostToDevice, m->dev->stream));
  FLOCK_TRY(enqueue_head(m, 0));
  FLOCK_CK(cudaMemcpyAsync(next_id, m->ids.p, 4, cudaMemcpyDeviceToHost, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_set_token(flock_model* m, int32_t id) {
  if (!m || id < 0 || id >= m->vocab) return FLOCK_E_ARG;
  FLOCK_CK(cudaMemcpyAsync(m->ids.p, &id, 4, cudaMemcpyHostToDevice, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

int flock_model_current_token(flock_model* m, int32_t* out) {
  FLOCK_CK(cudaMemcpyAsync(out, m->ids.p, 4, cudaMemcpyDeviceToHost, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

}  // extern "C"

// ============================================================ pipeline
//
// server/mesh.js:679 Flock.lap + web/bird.html:544 runFrame on one box: the
// coordinator rank (embedding, layers 0..cut-1, output_norm, head) sends the
// hidden state [n][hidden] to the next rank over NCCL, each stage runs its
// contiguous layer range and passes it on, the last stage sends it back to
// the coordinator, which projects the last row.  Every hop is stream-ordered
// on the GPUs; the host only sees the token id.

extern "C" {

int flock_comm_send_hidden(flock_comm* c, flock_model* m, int n_tokens, int peer) {
  if (!c || !m || n_tokens < 1 || n_tokens > m->ws.P) return FLOCK_E_ARG;
  FLOCK_TRY(comm_send(c, m->ws.h.p, (size_t)n_tokens * m->cfg.hidden, peer));
  return comm_wait(c);
}

int flock_comm_recv_hidden(flock_comm* c, flock_model* m, int n_tokens, int peer) {
  if (!c || !m || n_tokens < 1 || n_tokens > m->ws.P) return FLOCK_E_ARG;
  FLOCK_TRY(comm_recv(c, m->ws.h.p, (size_t)n_tokens * m->cfg.hidden, peer));
  return comm_wait(c);
}

int flock_pipeline_step(flock_model* m, flock_comm* c, const int32_t* ids, int n, int sync,
                        int32_t* next_id) {
  if (!m || n < 1 || n > m->cfg.max_prefill) {
    set_error("pipeline step of %d tokens: 1..maxPrefill %d", n, m ? m->cfg.max_prefill : 0);
    return FLOCK_E_ARG;
  }
  int rank = 0, nr = 1;
  if (c) FLOCK_TRY(comm_rank(c, &rank, &nr));
  FLOCK_CK(cudaSetDevice(m->dev->ordinal));
  FLOCK_TRY(check_room(m, n));
  const size_t nf = (size_t)n * m->cfg.hidden;
  if (rank == 0) {
    FLOCK_TRY(need_head(m));
    if (ids) FLOCK_TRY(upload_ids(m, ids, n));
    FLOCK_TRY(enqueue_embed(m, n));
    FLOCK_TRY(enqueue_layers(m, n));
    if (nr > 1) {
      FLOCK_TRY(comm_send(c, m->ws.h.p, nf, 1));
      FLOCK_TRY(comm_recv(c, m->ws.h.p, nf, nr - 1));
    }
    FLOCK_TRY(enqueue_head(m, n - 1));
    FLOCK_TRY(enqueue_record(m));
  } else {
    FLOCK_TRY(comm_recv(c, m->ws.h.p, nf, rank - 1));
    FLOCK_TRY(enqueue_layers(m, n));
    FLOCK_TRY(comm_send(c, m->ws.h.p, nf, (rank + 1) % nr));
  }
  m->pos += n;
  for (auto* L : m->layers) L->n_keys = m->pos;
  if (rank == 0 && next_id)
    FLOCK_CK(cudaMemcpyAsync(next_id, m->ids.p, 4, cudaMemcpyDeviceToHost, m->dev->stream));
  if (sync) return c ? comm_wait(c) : (cudaStreamSynchronize(m->dev->stream) == cudaSuccess
                                           ? FLOCK_OK : FLOCK_E_CUDA);
  return FLOCK_OK;
}

int flock_model_history(flock_model* m, int start, int n, int32_t* out) {
  if (!m || start < 0 || n < 0 || start + n > m->cfg.max_keys || (n && !out)) return FLOCK_E_ARG;
  if (n)
    FLOCK_CK(cudaMemcpyAsync(out, m->hist.as<int32_t>() + start, (size_t)n * 4,
                             cudaMemcpyDeviceToHost, m->dev->stream));
  FLOCK_TRY(sync_model(m));
  return check_device_errors(m);
}

}  // extern "C"

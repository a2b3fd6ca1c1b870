// Host side of the streaming persistent decode engine: builds each CTA's
// piece list (its row slices of every matrix, in consumption order, cut to
// ring slots), allocates the tagged exchange vectors and launches
// k_decode_stream cooperatively, one CTA per SM.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "decode_stream.cuh"
#include "stream_engine.h"

namespace flock {

StEngine::~StEngine() { delete args; }

namespace {

// Pieces of rows [r0, r1) of `a` (and the same rows of `b`, paired), cut to
// whole rows per ring slot; out0 = the output index of row r0.
void emit(std::vector<StPiece>& v, const flock_tensor* a, const flock_tensor* b, int64_t r0,
          int64_t r1, int64_t out0) {
  if (r1 <= r0) return;
  const int64_t K = a->cols;
  const int64_t scb = (int64_t)a->sc_stride * 2;
  const int64_t per = ST_SLOT / ((b ? 2 : 1) * (K + scb));
  for (int64_t r = r0; r < r1; r += per) {
    const int64_t n = std::min<int64_t>(per, r1 - r);
    StPiece p;
    std::memset(&p, 0, sizeof p);
    p.qs[0] = a->qs.as<uint8_t>() + r * K;
    p.sc[0] = a->sc.as<uint16_t>() + r * a->sc_stride;
    if (b) {
      p.qs[1] = b->qs.as<uint8_t>() + r * K;
      p.sc[1] = b->sc.as<uint16_t>() + r * b->sc_stride;
    }
    p.row_bytes = (uint32_t)K;
    p.sc_row = (uint16_t)scb;
    p.out_row = (uint32_t)(out0 + (r - r0));
    p.nrows = (uint16_t)n;
    p.flags = b ? ST_PAIR : 0;
    v.push_back(p);
  }
}

// Marks the end of a phase: its last piece, or an empty piece when this CTA
// has no rows in it (the consumer still sees the boundary).
void end_phase(std::vector<StPiece>& v, size_t start) {
  if (v.size() == start) {
    StPiece p;
    std::memset(&p, 0, sizeof p);
    v.push_back(p);
  }
  v.back().flags |= ST_LAST;
}

// CTA c's contiguous share of R rows over G CTAs.
void share(int64_t R, int c, int G, int64_t* r0, int64_t* r1) {
  *r0 = R * c / G;
  *r1 = R * (c + 1) / G;
}

// rows [r0, r1) of the concatenation of `ts` (each its own row count)
void emit_concat(std::vector<StPiece>& v, const flock_tensor* const* ts, int nt, int64_t r0,
                 int64_t r1) {
  int64_t off = 0;
  for (int i = 0; i < nt; i++) {
    const int64_t n = ts[i]->rows;
    const int64_t lo = std::max(r0, off), hi = std::min(r1, off + n);
    if (hi > lo) emit(v, ts[i], nullptr, lo - off, hi - off, lo);
    off += n;
  }
}

bool fits_slot(const flock_tensor* t, int mult) {
  return (int64_t)mult * (t->cols + (int64_t)t->sc_stride * 2) <= ST_SLOT;
}

}  // namespace

int stream_prepare(flock_dev* d, const StModelDesc& m, StEngine* e) {
  e->ok = false;
  auto no = [&](const char* why) {
    e->why = why;
    return FLOCK_OK;
  };
  if (m.hd != 128) return no("head_dim is not 128");
  if (m.nKV < 1 || m.nH % m.nKV || m.nH / m.nKV > ST_MAX_G) return no("GQA group above 4");
  if (m.n_layers < 1 || m.n_layers > 255) return no("layer count outside 1..255");
  if (!m.embd || !m.head || !m.out_norm) return no("no embedding/head");
  if (m.H % 32 || m.F % 32 || m.H > 8192 || m.F > 16384) return no("hidden/ffn shape");
  if (m.embd->dtype != FLOCK_Q8_0 || m.head->dtype != FLOCK_Q8_0) return no("head not Q8_0");
  for (int l = 0; l < m.n_layers; l++)
    for (int t = 0; t < 7; t++) {
      const flock_tensor* w = m.w[(size_t)l * W_COUNT + t];
      if (w->dtype != FLOCK_Q8_0) return no("a layer matrix is not Q8_0");
      if (!fits_slot(w, (t == W_GATE || t == W_UP) ? 2 : 1)) return no("row exceeds a ring slot");
    }
  if (m.head_in_kernel && !fits_slot(m.head, 1)) return no("head row exceeds a ring slot");
  int dev = d->ordinal, coop = 0, optin = 0;
  FLOCK_CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  FLOCK_CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (!coop) return no("no cooperative launch");
  int xbytes = 0;
  const size_t fixed = st_fixed_bytes(m.H, m.nH * m.hd, m.F, &xbytes);
  const size_t per_slot = st_smem_bytes(1, 0);
  const int64_t room = (int64_t)optin - (int64_t)fixed - 1024;
  int slots = room > 0 ? (int)(room / (int64_t)per_slot) : 0;
  if (slots < 4) return no("shared memory leaves fewer than 4 ring slots");
  if (slots > 32) slots = 32;  // one producer lane per slot
  const size_t smem = st_smem_bytes(slots, fixed);
  const int grid = d->sm_count;

  // piece lists: per CTA, per layer QKV | O | gate/up | down, then the head
  std::vector<std::vector<StPiece>> lists(grid);
  const int64_t qkv_rows = (int64_t)m.nH * m.hd + 2LL * m.nKV * m.hd;
  for (int c = 0; c < grid; c++) {
    auto& v = lists[c];
    int64_t r0, r1;
    for (int l = 0; l < m.n_layers; l++) {
      const flock_tensor* const* w = &m.w[(size_t)l * W_COUNT];
      size_t st = v.size();
      share(qkv_rows, c, grid, &r0, &r1);
      const flock_tensor* qkv[3] = {w[W_Q], w[W_K], w[W_V]};
      emit_concat(v, qkv, 3, r0, r1);
      end_phase(v, st);
      st = v.size();
      share(m.H, c, grid, &r0, &r1);
      emit(v, w[W_O], nullptr, r0, r1, r0);
      end_phase(v, st);
      st = v.size();
      share(m.F, c, grid, &r0, &r1);
      emit(v, w[W_GATE], w[W_UP], r0, r1, r0);
      end_phase(v, st);
      st = v.size();
      share(m.H, c, grid, &r0, &r1);
      emit(v, w[W_DOWN], nullptr, r0, r1, r0);
      end_phase(v, st);
    }
    if (m.head_in_kernel) {
      size_t st = v.size();
      share(m.head->rows, c, grid, &r0, &r1);
      emit(v, m.head, nullptr, r0, r1, r0);
      end_phase(v, st);
    }
  }
  size_t maxp = 0;
  for (auto& v : lists) maxp = std::max(maxp, v.size());
  std::vector<StPiece> table(maxp * grid);
  std::vector<int> counts(grid);
  for (int c = 0; c < grid; c++) {
    std::copy(lists[c].begin(), lists[c].end(), table.begin() + (size_t)c * maxp);
    counts[c] = (int)lists[c].size();
  }
  std::vector<StLayer> lt(m.n_layers);
  for (int l = 0; l < m.n_layers; l++) {
    const flock_tensor* const* w = &m.w[(size_t)l * W_COUNT];
    lt[l].attn_norm = w[W_ATTN_NORM]->data.as<float>();
    lt[l].q_norm = w[W_Q_NORM]->data.as<float>();
    lt[l].k_norm = w[W_K_NORM]->data.as<float>();
    lt[l].ffn_norm = w[W_FFN_NORM]->data.as<float>();
    lt[l].kcache = m.kcache[l];
    lt[l].vcache = m.vcache[l];
  }
  FLOCK_TRY(e->pieces.alloc(table.size() * sizeof(StPiece)));
  FLOCK_CK(cudaMemcpy(e->pieces.p, table.data(), table.size() * sizeof(StPiece),
                      cudaMemcpyHostToDevice));
  FLOCK_TRY(e->n_pieces.alloc(counts.size() * 4));
  FLOCK_CK(cudaMemcpy(e->n_pieces.p, counts.data(), counts.size() * 4, cudaMemcpyHostToDevice));
  FLOCK_TRY(e->layers.alloc(lt.size() * sizeof(StLayer)));
  FLOCK_CK(cudaMemcpy(e->layers.p, lt.data(), lt.size() * sizeof(StLayer), cudaMemcpyHostToDevice));
  // tagged vectors start at tag 0, which no launch uses (sequence >= 1)
  auto tagged = [&](DBuf& b, size_t words) -> int {
    FLOCK_TRY(b.alloc(words * 8));
    FLOCK_CK(cudaMemset(b.p, 0, words * 8));
    return FLOCK_OK;
  };
  FLOCK_TRY(tagged(e->t_qkv, (size_t)qkv_rows));
  FLOCK_TRY(tagged(e->t_part, (size_t)m.nH * ST_MAX_SPLITS * ST_PSTRIDE));
  FLOCK_TRY(tagged(e->t_att, (size_t)m.nH * m.hd));
  FLOCK_TRY(tagged(e->t_ho, (size_t)m.H));
  FLOCK_TRY(tagged(e->t_act, (size_t)m.F));
  FLOCK_TRY(tagged(e->t_hd, (size_t)m.H));
  FLOCK_TRY(e->seq.alloc(16));
  const unsigned one = 1;
  FLOCK_CK(cudaMemset(e->seq.p, 0, 16));
  FLOCK_CK(cudaMemcpy(e->seq.p, &one, 4, cudaMemcpyHostToDevice));
  FLOCK_TRY(e->err.alloc(16));
  FLOCK_CK(cudaMemset(e->err.p, 0, 16));
  FLOCK_TRY(e->am_val.alloc((size_t)grid * 4));
  FLOCK_TRY(e->am_idx.alloc((size_t)grid * 4));
  FLOCK_TRY(e->am_count.alloc(16));
  FLOCK_CK(cudaMemset(e->am_count.p, 0, 16));

  // RoPE (cos, sin) for every position the cache holds
  const int rope_rows = std::max(1, m.max_keys);
  FLOCK_TRY(e->rope.alloc((size_t)rope_rows * 64 * sizeof(float2)));
  k_rope_table<<<(rope_rows * 64 + 255) / 256, 256>>>(m.inv_freq, rope_rows, e->rope.as<float2>());
  FLOCK_CK(cudaGetLastError());
  FLOCK_CK(cudaDeviceSynchronize());
  if (!e->args) e->args = new StArgs();
  StArgs& a = *e->args;
  a = StArgs{};
  a.layers = e->layers.as<StLayer>();
  a.n_layers = m.n_layers;
  a.H = m.H;
  a.nH = m.nH;
  a.nKV = m.nKV;
  a.hd = m.hd;
  a.F = m.F;
  a.vocab = m.vocab;
  a.kv_bf16 = m.kv_bf16;
  a.eps = m.eps;
  a.neox = m.neox;
  a.inv_freq = m.inv_freq;
  a.rope_cs = e->rope.as<float2>();
  a.rope_rows = rope_rows;
  a.embd_qs = m.embd->qs.as<uint8_t>();
  a.embd_sc = m.embd->sc.as<uint16_t>();
  a.embd_sc_stride = m.embd->sc_stride;
  a.out_norm = m.out_norm->data.as<float>();
  a.pieces = e->pieces.as<StPiece>();
  a.n_pieces = e->n_pieces.as<int>();
  a.max_pieces = (int)maxp;
  a.t_qkv = e->t_qkv.as<uint64_t>();
  a.t_part = e->t_part.as<uint64_t>();
  a.t_att = e->t_att.as<uint64_t>();
  a.t_ho = e->t_ho.as<uint64_t>();
  a.t_act = e->t_act.as<uint64_t>();
  a.t_hd = e->t_hd.as<uint64_t>();
  a.h_out = m.h_out;
  a.logits = m.logits;
  a.ids = m.ids;
  a.hist = m.hist;
  a.hist_cap = m.hist_cap;
  a.ctl = m.ctl;
  a.seq = e->seq.as<unsigned>();
  a.am_val = e->am_val.as<float>();
  a.am_idx = e->am_idx.as<uint32_t>();
  a.am_count = e->am_count.as<uint32_t>();
  a.err = e->err.as<int>();
  a.trace = nullptr;
  a.splits_max = std::max(1, std::min(ST_MAX_SPLITS, grid / m.nKV));
  a.head = m.head_in_kernel ? 1 : 0;
  a.l2_rounds = 3;
  a.ring_slots = slots;
  a.xbytes = xbytes;
  const void* kfn = m.H <= 1024 ? (const void*)k_decode_stream<true>
                                 : (const void*)k_decode_stream<false>;
  FLOCK_TRY(kernel_setup(kfn, (int)smem));
  int per_sm = 0;
  FLOCK_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, ST_THREADS,
                                                         smem));
  if (per_sm < 1) return no("the kernel does not fit an SM");
  e->smem = smem;
  e->grid = grid;
  e->n_layers = m.n_layers;
  e->ok = true;
  return FLOCK_OK;
}

int stream_launch(StEngine* e, cudaStream_t st) {
  if (!e->ok) {
    set_error("streaming decode engine unavailable: %s", e->why.c_str());
    return FLOCK_E_UNSUPPORTED;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(e->grid);
  cfg.blockDim = dim3(ST_THREADS);
  cfg.dynamicSmemBytes = e->smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (e->args->H <= 1024)
    FLOCK_CK(cudaLaunchKernelEx(&cfg, k_decode_stream<true>, *e->args));
  else
    FLOCK_CK(cudaLaunchKernelEx(&cfg, k_decode_stream<false>, *e->args));
  return FLOCK_OK;
}

int stream_check(StEngine* e) {
  if (!e || !e->ok) return FLOCK_OK;
  int err = 0;
  FLOCK_CK(cudaMemcpy(&err, e->err.p, 4, cudaMemcpyDeviceToHost));
  if (err) {
    set_error("streaming decode kernel gave up waiting (%s)",
              err == ST_ERR_RING ? "weight ring" : "exchange vector");
    cudaMemset(e->err.p, 0, 4);
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

int stream_trace_stride(const StEngine* e) { return st_trace_stride(e->n_layers); }

int stream_trace(StEngine* e, bool enable) {
  if (!e->ok) return FLOCK_E_UNSUPPORTED;
  if (enable && !e->trace.p) {
    const size_t n = (size_t)e->grid * st_trace_stride(e->n_layers);
    FLOCK_TRY(e->trace.alloc(n * 8));
    FLOCK_CK(cudaMemset(e->trace.p, 0, n * 8));
  }
  e->args->trace = enable ? e->trace.as<unsigned long long>() : nullptr;
  return FLOCK_OK;
}

}  // namespace flock

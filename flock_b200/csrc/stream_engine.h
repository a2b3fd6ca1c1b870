// Host side of the streaming persistent decode engine (k_decode_stream,
// decode_stream.cuh): the per-CTA weight piece lists, the tagged exchange
// vectors and the launch.  Internal to libflock_cuda.so.
#pragma once
#include <string>
#include <vector>

#include "flock_internal.h"

namespace flock {

struct StArgs;

// What a model hands the engine: its shape, tensors and the device buffers
// the step reads and writes (all owned by the model).
struct StModelDesc {
  int H = 0, nH = 0, nKV = 0, hd = 0, F = 0, vocab = 0, n_layers = 0;
  float eps = 0.0f;
  int neox = 1;
  int kv_bf16 = 0;
  std::vector<const flock_tensor*> w;  // [n_layers][W_COUNT]
  const flock_tensor* embd = nullptr;
  const flock_tensor* head = nullptr;
  const flock_tensor* out_norm = nullptr;
  const float* inv_freq = nullptr;  // device [hd / 2]
  std::vector<void*> kcache, vcache;  // [n_layers]
  float* h_out = nullptr;   // [H]
  float* logits = nullptr;  // [vocab]
  int32_t* ids = nullptr;
  int32_t* hist = nullptr;
  int hist_cap = 0;
  int max_keys = 0;  // positions the RoPE table covers
  // true: the LM head and its argmax run inside the streaming kernel; false:
  // the kernel ends with the last layer's hidden state (h_out) and the caller
  // launches the head GEMV (the kernel still advances the position)
  bool head_in_kernel = false;
  int* ctl = nullptr;
};

struct StEngine {
  bool ok = false;
  std::string why;  // why the engine is unavailable for this model
  StArgs* args = nullptr;
  DBuf layers, pieces, n_pieces, t_qkv, t_part, t_att, t_ho, t_act, t_hd, seq, err, am_val,
      am_idx, am_count, trace, rope;
  size_t smem = 0;
  int grid = 0;
  int n_layers = 0;
  ~StEngine();
};

// Builds the engine for `m` on device `d` (current).  Returns FLOCK_OK with
// e->ok false (and e->why set) when the shape does not fit the engine.
int stream_prepare(flock_dev* d, const StModelDesc& m, StEngine* e);
// One decode step (one cooperative launch) on `st`.
int stream_launch(StEngine* e, cudaStream_t st);
// FLOCK_E_CUDA (and the error word cleared) if a wait gave up since the last
// check; call after a synchronisation.
int stream_check(StEngine* e);
// Phase trace on/off (per CTA, st_trace_stride(n_layers) words per token).
int stream_trace(StEngine* e, bool enable);
int stream_trace_stride(const StEngine* e);

}  // namespace flock

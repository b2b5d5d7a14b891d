// C ABI of the wave-MCTS engine (declarations and reference map in include/omq_b200.h).
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>

#include "omq_internal.cuh"

namespace omq {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return OMQ_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return OMQ_CUDA_ERROR;
}

static std::atomic<unsigned long long> g_launches{0};

void count_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace omq

using namespace omq;

#define OMQ_CHECK_LAUNCH(what)                                          \
  do {                                                                  \
    cudaError_t _e = cudaGetLastError();                                \
    if (_e != cudaSuccess) return cuda_status(_e, what);                \
  } while (0)

extern "C" {

const char* omq_status_string(int s) {
  switch (s) {
    case OMQ_OK: return "ok";
    case OMQ_TREE_FULL: return "tree full";
    case OMQ_QUEUE_OVERFLOW: return "queue overflow";
    case OMQ_TIMEOUT: return "timeout";
    case OMQ_BAD_ARG: return "bad argument";
    case OMQ_CUDA_ERROR: return "cuda error";
    case OMQ_NOT_READY: return "phase called out of order";
    default: return "unknown status";
  }
}

const char* omq_last_error(void) { return g_err; }

int omq_abi_struct_sizes(uint32_t* h_engine_config, uint32_t* h_resnet_config) {
  if (!h_engine_config || !h_resnet_config) { set_error("null argument"); return OMQ_BAD_ARG; }
  *h_engine_config = (uint32_t)sizeof(omq_engine_config);
  *h_resnet_config = (uint32_t)sizeof(omq_resnet_config);
  return OMQ_OK;
}

int omq_kernel_launches_add(int64_t delta) {
  g_launches.fetch_add((unsigned long long)delta, std::memory_order_relaxed);
  return OMQ_OK;
}

int omq_kernel_launches(uint64_t* h_count) {
  if (!h_count) { set_error("null argument"); return OMQ_BAD_ARG; }
  *h_count = g_launches.load();
  return OMQ_OK;
}

int omq_engine_create(const omq_engine_config* cfg, omq_engine** out) {
  if (!cfg || !out) { set_error("null argument"); return OMQ_BAD_ARG; }
  *out = nullptr;
  const omq_engine_config c = *cfg;
  if (c.game == OMQ_GAME_GO && c.go_superko && c.go_cycle) {
    set_error("go_superko and go_cycle are exclusive (Chinese vs Japanese / Korean rules)");
    return OMQ_BAD_ARG;
  }
  if (c.dirichlet_epsilon > 0 && !(c.dirichlet_alpha > 0)) {
    set_error("dirichlet_alpha must be > 0 when dirichlet_epsilon > 0");
    return OMQ_BAD_ARG;
  }
  if (c.num_trees < 1 || c.board_size < (c.game == OMQ_GAME_CHESS ? 8 : 5) || c.board_size > 19 || c.capacity < 2 ||
      c.max_wave_size < 1 || c.max_wave_size > 1024 || c.max_depth < 2 || c.max_depth > 127 ||
      (c.game != OMQ_GAME_GOMOKU && c.game != OMQ_GAME_GO && c.game != OMQ_GAME_CHESS) ||
      (c.game == OMQ_GAME_CHESS && c.board_size != 8)) {
    set_error("bad engine config: trees=%d board=%d capacity=%d wave=%d depth=%d game=%d",
              c.num_trees, c.board_size, c.capacity, c.max_wave_size, c.max_depth, c.game);
    return OMQ_BAD_ARG;
  }
  DeviceGuard g(c.device);
  omq_engine* e = new (std::nothrow) omq_engine();
  if (!e) { set_error("host allocation failed"); return OMQ_BAD_ARG; }
  e->cfg = c;
  EngineView& v = e->v;
  v.R = c.num_trees;
  v.T = c.capacity;
  v.S = c.board_size;
  v.C = c.board_size * c.board_size;
  v.game = c.game;
  v.A = c.game == OMQ_GAME_GO ? v.C + 1 : c.game == OMQ_GAME_CHESS ? 4672 : v.C;
  v.max_children = c.game == OMQ_GAME_CHESS ? 256 : v.A;
  v.WCAP = c.max_wave_size;
  v.LOGCAP = c.max_wave_size * c.max_depth;
  v.max_depth = c.max_depth;
  v.enable_vl = c.enable_virtual_loss ? 1 : 0;
  v.c_puct = c.c_puct;
  v.vl_value = -(c.virtual_loss < 0 ? -c.virtual_loss : c.virtual_loss);
  v.noise_alpha = c.dirichlet_alpha;
  v.noise_eps = c.dirichlet_epsilon > 0 ? c.dirichlet_epsilon : 0.0f;
  v.noise_keep = (float)(1.0 - (double)v.noise_eps);
  v.noise_seed = c.noise_seed;
  v.go_superko = (c.game == OMQ_GAME_GO && c.go_superko) ? 1 : 0;
  v.go_cycle = (c.game == OMQ_GAME_GO && c.go_cycle) ? 1 : 0;
  // few trees: several CTAs (SMs) per tree in selection and expansion (4 trees or fewer per 148 SMs
  // get up to 8 each)
  {
    int sms = 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c.device) != cudaSuccess || sms <= 0) {
      cudaGetLastError();
      sms = 148;
    }
    v.slices = 4 * v.R <= sms ? std::max(1, std::min(8, sms / (2 * v.R))) : 1;
  }
  const size_t R = v.R, T = v.T, W = v.WCAP, QC = R * W;
  size_t off[40], n = 0, tot = 0;
  auto take = [&](size_t bytes) { off[n++] = tot; tot += align256(bytes); };
  take(R * T * sizeof(NodeStats));            // 0 stats
  take(R * T * sizeof(NodeTopo));             // 1 topo
  const bool chess = c.game == OMQ_GAME_CHESS;
  take(chess ? R * 101 * 80 : R * v.C * (c.game == OMQ_GAME_GO ? 8 : 1));  // 2 roots (+ history)
  take(R * sizeof(TreeHeader));               // 3 headers
  take(R * v.slices * 2 * W * sizeof(Visit)); // 4 frontier (per slice)
  take(R * (size_t)v.LOGCAP * sizeof(Visit)); // 5 visit log
  take(R * W * sizeof(Visit));                // 6 leaves
  take(R * W * sizeof(int2));                 // 7 leaf_final
  take(R * W * sizeof(float));                // 8 simval
  take(QC * sizeof(int2));                    // 9 q entries expand
  take(QC * sizeof(int2));                    // 10 q entries final
  take(QC * (size_t)v.A * sizeof(float));     // 11 policy expand
  take(QC * (size_t)v.A * sizeof(float));     // 12 policy final
  take(QC * sizeof(float));                   // 13 value expand
  take(QC * sizeof(float));                   // 14 value final
  take(2 * sizeof(int32_t));                  // 15 counts
  take(R * (size_t)v.A * sizeof(float));      // 16 root noise
  take(c.game == OMQ_GAME_GO ? R * W * 32 * sizeof(uint32_t)
       : chess ? R * W * 148 * sizeof(uint32_t) : 16);                    // 17 per-leaf legal masks
  take(chess ? R * 100 * sizeof(uint64_t) : 16);                          // 18 chess prior hashes
  take(c.game == OMQ_GAME_GO ? R * OMQ_GO_MAX_KEYS * sizeof(uint64_t) : 16);  // 19 Go superko keys
  take(c.game == OMQ_GAME_GO ? R * 128 * sizeof(uint32_t) : 16);              // 20 Go key filter
  take(c.game == OMQ_GAME_GOMOKU ? R * W * 128 * sizeof(int16_t) : 16);       // 21 leaf paths
  take(R * 4 * sizeof(int32_t));                                              // 22 select counters
  void* arena = nullptr;
  cudaError_t err = cudaMalloc(&arena, tot);
  if (err != cudaSuccess) {
    delete e;
    return cuda_status(err, "cudaMalloc(engine arena)");
  }
  char* b = static_cast<char*>(arena);
  v.stats = reinterpret_cast<NodeStats*>(b + off[0]);
  v.topo = reinterpret_cast<NodeTopo*>(b + off[1]);
  v.root_board = reinterpret_cast<int8_t*>(b + off[2]);
  v.hdr = reinterpret_cast<TreeHeader*>(b + off[3]);
  v.frontier = reinterpret_cast<Visit*>(b + off[4]);
  v.vlog = reinterpret_cast<Visit*>(b + off[5]);
  v.leaves = reinterpret_cast<Visit*>(b + off[6]);
  v.leaf_final = reinterpret_cast<int2*>(b + off[7]);
  v.simval = reinterpret_cast<float*>(b + off[8]);
  v.q_entries[0] = reinterpret_cast<int2*>(b + off[9]);
  v.q_entries[1] = reinterpret_cast<int2*>(b + off[10]);
  v.q_policy[0] = reinterpret_cast<float*>(b + off[11]);
  v.q_policy[1] = reinterpret_cast<float*>(b + off[12]);
  v.q_value[0] = reinterpret_cast<float*>(b + off[13]);
  v.q_value[1] = reinterpret_cast<float*>(b + off[14]);
  v.q_count = reinterpret_cast<int32_t*>(b + off[15]);
  v.root_noise = reinterpret_cast<float*>(b + off[16]);
  v.go_mask = reinterpret_cast<uint32_t*>(b + off[17]);
  v.chess_prior_hash = reinterpret_cast<uint64_t*>(b + off[18]);
  v.go_keys = reinterpret_cast<uint64_t*>(b + off[19]);
  v.go_bloom = reinterpret_cast<uint32_t*>(b + off[20]);
  v.leaf_paths = reinterpret_cast<int16_t*>(b + off[21]);
  v.sel_ctr = reinterpret_cast<int32_t*>(b + off[22]);
  err = cudaMemset(v.hdr, 0, R * sizeof(TreeHeader));
  if (err == cudaSuccess) err = cudaMemset(v.q_count, 0, 2 * sizeof(int32_t));
  if (err == cudaSuccess) err = cudaMemset(v.root_noise, 0, R * (size_t)v.A * sizeof(float));
  if (err != cudaSuccess) {
    cudaFree(arena);
    delete e;
    return cuda_status(err, "cudaMemset(engine)");
  }
  e->arena = arena;
  e->bytes = tot;
  e->phase = 0;
  *out = e;
  return OMQ_OK;
}

int omq_engine_destroy(omq_engine* e) {
  if (!e) return OMQ_OK;
  DeviceGuard g(e->cfg.device);
  cudaError_t err = cudaFree(e->arena);
  if (e->reroot_scratch) {
    const cudaError_t e2 = cudaFree(e->reroot_scratch);
    if (err == cudaSuccess) err = e2;
  }
  delete e;
  return cuda_status(err, "cudaFree(engine arena)");
}

int omq_engine_memory(const omq_engine* e, uint64_t* bytes) {
  if (!e || !bytes) { set_error("null argument"); return OMQ_BAD_ARG; }
  *bytes = e->bytes;
  return OMQ_OK;
}

int omq_reroot(omq_engine* e, const int32_t* d_actions, int mode, void* stream) {
  if (!e || !d_actions) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (mode != OMQ_REROOT_CARRY && mode != OMQ_REROOT_KEEP) {
    set_error("omq_reroot mode %d (OMQ_REROOT_CARRY or OMQ_REROOT_KEEP)", mode);
    return OMQ_BAD_ARG;
  }
  if (e->phase == 1 || e->phase == 3 || e->phase == 4) {
    set_error("omq_reroot between searches only (a search is in progress)");
    return OMQ_NOT_READY;
  }
  DeviceGuard g(e->cfg.device);
  NodeStats* ss = nullptr;
  NodeTopo* st = nullptr;
  if (mode == OMQ_REROOT_KEEP) {
    const size_t per_tree = (size_t)e->v.T * (sizeof(NodeStats) + sizeof(NodeTopo));
    if (!e->reroot_scratch) {
      // node copies for a chunk of trees, about 1 GiB at most (at least one tree)
      const size_t chunk = std::max<size_t>(1, std::min<size_t>(e->v.R, (size_t(1) << 30) / per_tree));
      void* p = nullptr;
      const cudaError_t err = cudaMalloc(&p, chunk * per_tree);
      if (err != cudaSuccess) return cuda_status(err, "cudaMalloc(reroot scratch)");
      e->reroot_scratch = p;
      e->reroot_chunk = (int32_t)chunk;
      e->bytes += chunk * per_tree;
    }
    ss = static_cast<NodeStats*>(e->reroot_scratch);
    st = reinterpret_cast<NodeTopo*>(static_cast<char*>(e->reroot_scratch) +
                                     (size_t)e->reroot_chunk * e->v.T * sizeof(NodeStats));
  }
  launch_reroot(e->v, d_actions, mode, ss, st, e->reroot_chunk > 0 ? e->reroot_chunk : e->v.R,
                (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_reroot");
  e->phase = 0;
  return OMQ_OK;
}

int omq_begin(omq_engine* e, const int8_t* d_boards, void* stream) {
  if (!e || !d_boards) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (e->v.game != OMQ_GAME_GOMOKU) {
    set_error("omq_begin is for Gomoku engines (omq_begin_go / omq_begin_chess)");
    return OMQ_BAD_ARG;
  }
  DeviceGuard g(e->cfg.device);
  launch_begin(e->v, d_boards, e->searches++, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_begin");
  e->phase = 1;
  return OMQ_OK;
}

int omq_begin_chess(omq_engine* e, const void* d_records, const int32_t* d_nprior, void* stream) {
  if (!e || !d_records || !d_nprior) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (e->v.game != OMQ_GAME_CHESS) { set_error("omq_begin_chess on a non-chess engine"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  launch_begin_chess(e->v, d_records, d_nprior, e->searches++, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_begin_chess");
  e->phase = 1;
  return OMQ_OK;
}

int omq_begin_go(omq_engine* e, const int8_t* d_history, const int32_t* d_meta,
                 const uint64_t* d_keys, const int32_t* d_nkeys, void* stream) {
  if (!e || !d_history || !d_meta) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (e->v.game != OMQ_GAME_GO) { set_error("omq_begin_go on a non-Go engine"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  launch_begin_go(e->v, d_history, d_meta, d_nkeys ? d_keys : nullptr, d_keys ? d_nkeys : nullptr,
                  e->searches++, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_begin_go");
  e->phase = 1;
  return OMQ_OK;
}

int omq_root_expand(omq_engine* e, void* stream) {
  if (!e) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (e->phase != 1) { set_error("omq_root_expand before omq_begin"); return OMQ_NOT_READY; }
  DeviceGuard g(e->cfg.device);
  launch_expand(e->v, 1, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_root_expand");
  e->phase = 2;
  return OMQ_OK;
}

int omq_wave_select(omq_engine* e, int32_t wave, void* stream) {
  if (!e) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (e->phase != 2) { set_error("omq_wave_select needs an expanded root / finished wave"); return OMQ_NOT_READY; }
  if (wave < 1 || wave > e->v.WCAP) { set_error("wave size %d outside [1, %d]", wave, e->v.WCAP); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  launch_select(e->v, wave, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_wave_select");
  e->wave = wave;
  e->phase = 3;
  return OMQ_OK;
}

int omq_wave_expand(omq_engine* e, void* stream) {
  if (!e) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (e->phase != 3) { set_error("omq_wave_expand before omq_wave_select"); return OMQ_NOT_READY; }
  DeviceGuard g(e->cfg.device);
  launch_expand(e->v, 0, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_wave_expand");
  e->phase = 4;
  return OMQ_OK;
}

int omq_wave_backup(omq_engine* e, void* stream) {
  if (!e) { set_error("null argument"); return OMQ_BAD_ARG; }
  if (e->phase != 4) { set_error("omq_wave_backup before omq_wave_expand"); return OMQ_NOT_READY; }
  DeviceGuard g(e->cfg.device);
  launch_backup(e->v, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_wave_backup");
  e->phase = 2;
  return OMQ_OK;
}

int omq_queue_buffers(omq_engine* e, int32_t queue, int32_t** d_entries, float** d_policy,
                      float** d_value, int32_t** d_count, int32_t* h_capacity) {
  if (!e || queue < 0 || queue > 1) { set_error("bad queue"); return OMQ_BAD_ARG; }
  if (d_entries) *d_entries = reinterpret_cast<int32_t*>(e->v.q_entries[queue]);
  if (d_policy) *d_policy = e->v.q_policy[queue];
  if (d_value) *d_value = e->v.q_value[queue];
  if (d_count) *d_count = e->v.q_count + queue;
  if (h_capacity) *h_capacity = e->v.R * e->v.WCAP;
  return OMQ_OK;
}

int omq_queue_count(omq_engine* e, int32_t queue, int32_t* h_count, void* stream) {
  if (!e || !h_count || queue < 0 || queue > 1) { set_error("bad queue"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t err = cudaMemcpyAsync(h_count, e->v.q_count + queue, sizeof(int32_t),
                                    cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  return cuda_status(err, "omq_queue_count");
}

int omq_queue_features(omq_engine* e, int32_t queue, float* d_out, void* stream) {
  if (!e || !d_out || queue < 0 || queue > 1) { set_error("bad argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  launch_features(e->v, queue, d_out, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_queue_features");
  return OMQ_OK;
}

int omq_queue_eval_synthetic(omq_engine* e, int32_t queue, void* stream) {
  if (!e || queue < 0 || queue > 1) { set_error("bad queue"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  launch_synth_eval(e->v, queue, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_queue_eval_synthetic");
  return OMQ_OK;
}

int omq_root_noise(omq_engine* e, float* d_noise, void* stream) {
  if (!e || !d_noise) { set_error("null argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  return cuda_status(cudaMemcpyAsync(d_noise, e->v.root_noise, sizeof(float) * e->v.R * e->v.A,
                                     cudaMemcpyDeviceToDevice, (cudaStream_t)stream),
                     "omq_root_noise");
}

int omq_tree_status(omq_engine* e, int32_t* d_status, int32_t* d_num_nodes, void* stream) {
  if (!e) { set_error("null argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  launch_status(e->v, d_status, d_num_nodes, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_tree_status");
  return OMQ_OK;
}

static int first_tree_status(omq_engine* e, cudaStream_t s) {
  TreeHeader* h = new (std::nothrow) TreeHeader[e->v.R];
  if (!h) { set_error("host allocation failed"); return OMQ_BAD_ARG; }
  cudaError_t err = cudaMemcpyAsync(h, e->v.hdr, sizeof(TreeHeader) * e->v.R,
                                    cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  int st = cuda_status(err, "reading tree status");
  for (int r = 0; st == OMQ_OK && r < e->v.R; ++r)
    if (h[r].status != OMQ_OK) {
      st = h[r].status;
      set_error("tree %d: %s (%d nodes of %d)", r, omq_status_string(st), h[r].num_nodes, e->v.T);
    }
  delete[] h;
  return st;
}

// Leaf evaluator of a one-call search: the built-in synthetic evaluator (net == nullptr) or a
// tensor-core ResNet reading the engine's leaf queue in place.
static int eval_queue(omq_engine* e, omq_resnet* net, int queue, void* stream) {
  return net ? omq_resnet_forward_queue(net, e, queue, stream) : omq_queue_eval_synthetic(e, queue, stream);
}

// Root expansion and ceil(sims / max_wave_size) waves (MCTS._run_search, mcts.py:1020-1063), every
// evaluation through the on-device leaf queues; one host synchronisation at the end (tree status).
static int search_waves(omq_engine* e, omq_resnet* net, int32_t sims, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  int st;
  if ((st = eval_queue(e, net, OMQ_QUEUE_EXPAND, stream))) return st;
  if ((st = omq_root_expand(e, stream))) return st;
  for (int done = 0; done < sims;) {
    const int w = sims - done < e->v.WCAP ? sims - done : e->v.WCAP;
    if ((st = omq_wave_select(e, w, stream))) return st;
    if ((st = eval_queue(e, net, OMQ_QUEUE_EXPAND, stream))) return st;
    if ((st = omq_wave_expand(e, stream))) return st;
    if ((st = eval_queue(e, net, OMQ_QUEUE_FINAL, stream))) return st;
    if ((st = omq_wave_backup(e, stream))) return st;
    done += w;
  }
  DeviceGuard g(e->cfg.device);
  return first_tree_status(e, s);
}

int omq_search_synthetic(omq_engine* e, const int8_t* d_boards, int32_t sims, void* stream) {
  return omq_search(e, nullptr, d_boards, sims, stream);
}

int omq_search_synthetic_chess(omq_engine* e, const void* d_records, const int32_t* d_nprior,
                               int32_t sims, void* stream) {
  return omq_search_chess(e, nullptr, d_records, d_nprior, sims, stream);
}

int omq_search_synthetic_go(omq_engine* e, const int8_t* d_history, const int32_t* d_meta,
                            const uint64_t* d_keys, const int32_t* d_nkeys, int32_t sims, void* stream) {
  return omq_search_go(e, nullptr, d_history, d_meta, d_keys, d_nkeys, sims, stream);
}

int omq_search(omq_engine* e, omq_resnet* net, const int8_t* d_boards, int32_t sims, void* stream) {
  if (!e || !d_boards || sims < 0) { set_error("bad argument"); return OMQ_BAD_ARG; }
  int st = omq_begin(e, d_boards, stream);
  if (st) return st;
  return search_waves(e, net, sims, stream);
}

int omq_search_go(omq_engine* e, omq_resnet* net, const int8_t* d_history, const int32_t* d_meta,
                  const uint64_t* d_keys, const int32_t* d_nkeys, int32_t sims, void* stream) {
  if (!e || !d_history || !d_meta || sims < 0) { set_error("bad argument"); return OMQ_BAD_ARG; }
  int st = omq_begin_go(e, d_history, d_meta, d_keys, d_nkeys, stream);
  if (st) return st;
  return search_waves(e, net, sims, stream);
}

int omq_search_chess(omq_engine* e, omq_resnet* net, const void* d_records, const int32_t* d_nprior,
                     int32_t sims, void* stream) {
  if (!e || !d_records || !d_nprior || sims < 0) { set_error("bad argument"); return OMQ_BAD_ARG; }
  int st = omq_begin_chess(e, d_records, d_nprior, stream);
  if (st) return st;
  return search_waves(e, net, sims, stream);
}

int omq_root_visits(omq_engine* e, int32_t* d_visits, float* d_root_nw, void* stream) {
  if (!e || !d_visits) { set_error("null argument"); return OMQ_BAD_ARG; }
  DeviceGuard g(e->cfg.device);
  launch_root_visits(e->v, d_visits, d_root_nw, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_root_visits");
  return OMQ_OK;
}

int omq_selftest_prior_sum(const float* d_x, const int32_t* d_offsets, int32_t segments, float* d_out,
                           void* stream) {
  if (!d_x || !d_offsets || !d_out || segments < 0) { set_error("bad argument"); return OMQ_BAD_ARG; }
  if (segments == 0) return OMQ_OK;
  launch_selftest_prior_sum(d_x, d_offsets, segments, d_out, (cudaStream_t)stream);
  return cuda_status(cudaGetLastError(), "k_selftest_prior_sum");
}

int omq_export_tree(omq_engine* e, int32_t tree, int32_t count, int32_t* N, float* W, float* P,
                    int32_t* VL, int32_t* parent, int32_t* action, uint8_t* terminal,
                    void* stream) {
  if (!e || tree < 0 || tree >= e->v.R || count < 0 || count > e->v.T) {
    set_error("bad export arguments");
    return OMQ_BAD_ARG;
  }
  if (count == 0) return OMQ_OK;
  DeviceGuard g(e->cfg.device);
  launch_export(e->v, tree, count, N, W, P, VL, parent, action, terminal, (cudaStream_t)stream);
  OMQ_CHECK_LAUNCH("omq_export_tree");
  return OMQ_OK;
}

}  // extern "C"

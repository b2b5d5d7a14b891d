// Parity oracle - TEST INFRASTRUCTURE ONLY. See oracle.h for the reference map.
//
// The wave is restated literally, one simulation at a time, in the reference's order. All
// arithmetic is fp32 with one rounding per operation (built with -ffp-contract=off), in the
// operand order the reference's torch expressions evaluate.
#include "oracle.h"
#include "torch_sum.h"
#include "chess_rules.h"
#include "go_rules.h"
#include "gomoku_rules.h"
#include "synth_eval.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <vector>

namespace {

struct Tree {
  int cap, size, cells, actions;
  oracle_config cfg{};
  oracle_eval_fn eval = nullptr;
  void* ctx = nullptr;
  int num_nodes = 0;
  std::vector<int32_t> N, VL, parent, action, child_start, child_count, mc;
  std::vector<float> W, P;
  std::vector<uint8_t> terminal;
  std::vector<int8_t> player, boards;
  oracle_result res{};
  std::vector<float> feat, pol, val;
  std::vector<float> root_noise;  // by action, for the next wave only
  float noise_eps = 0.0f, noise_keep = 1.0f;

  // Go (game == 1): actions = cells + 1 (pass last); per-node ko point and consecutive passes;
  // positions before the root come from root_hist[1..7].
  int game = 0, planes = oracle::kPlanes;
  std::vector<int32_t> ko, passes;
  std::vector<int8_t> root_hist;
  // Go positional superko: the game's keys before the root, and each node's key (board + ko)
  int superko = 0, cycle = 0;
  std::vector<uint64_t> root_keys, node_key;
  // Chess (game == 2): a position record per node, the game's positions before the root (most
  // recent first) for the history planes and the repetition count.
  std::vector<oracle_chess_pos> cpos, prior;
  // Subtree reuse between searches (reroot): 0 fresh tree, 1 fresh tree whose root starts with
  // (carry_n, carry_w), 2 nodes [0, num_nodes) are the kept subtree of the next root.
  int kept = 0;
  int32_t carry_n = 0;
  float carry_w = 0.f;

  // Root child reached by move a becomes the next search's root. Mode 1: the reference's
  // use_gpu_tree_reuse path (mcts.py:1929-2005) observably keeps the child's visit count and value
  // sum on a fresh root. Mode 2: the child's subtree as CSRTree.shift_root describes it
  // (csr_tree.py:1020-1229): breadth-first order, children in action order, per-node data moved
  // with the nodes. A child without children falls back to mode 1.
  int reroot(int a, int mode) {
    kept = 0;
    if (num_nodes < 1 || res.status != 0 || a < 0) return 0;
    int c = -1;
    for (int j = 0; j < child_count[0]; ++j)
      if (action[child_start[0] + j] == a) c = child_start[0] + j;
    if (c < 0) return 0;
    if (mode == 1 || child_count[c] == 0) {
      kept = 1; carry_n = N[c]; carry_w = W[c];
      return 1;
    }
    std::vector<int> order{c}, ncs{0}, npar{-1};
    for (size_t i = 0; i < order.size(); ++i) {
      const int o = order[i];
      ncs[i] = child_count[o] ? (int)order.size() : 0;
      for (int j = 0; j < child_count[o]; ++j) {
        order.push_back(child_start[o] + j);
        ncs.push_back(0);
        npar.push_back((int)i);
      }
    }
    const int k = (int)order.size();
    auto perm = [&](auto& vec, size_t width) {
      if (vec.size() < (size_t)k * width) return;
      auto old = vec;
      for (int i = 0; i < k; ++i)
        for (size_t w = 0; w < width; ++w) vec[(size_t)i * width + w] = old[(size_t)order[i] * width + w];
    };
    perm(N, 1); perm(VL, 1); perm(W, 1); perm(P, 1); perm(terminal, 1); perm(player, 1); perm(mc, 1);
    perm(ko, 1); perm(passes, 1); perm(boards, (size_t)cells); perm(action, 1); perm(child_count, 1);
    if (!node_key.empty()) perm(node_key, 1);
    if (!cpos.empty()) perm(cpos, 1);
    for (int i = 0; i < k; ++i) { child_start[i] = ncs[i]; parent[i] = npar[i]; }
    action[0] = -1;
    num_nodes = k;
    kept = 2;
    return 2;
  }

  // Node 0 and the node count for a new search; returns true when the kept subtree stays (its
  // root is already expanded: no forced root expansion).
  bool install_root() {
    const int k = kept;
    kept = 0;
    if (k == 2) return true;
    num_nodes = 1;
    N[0] = k == 1 ? carry_n : 0; W[0] = k == 1 ? carry_w : 0.f;
    VL[0] = 0; P[0] = 1.0f; parent[0] = -1; action[0] = -1;
    child_count[0] = 0;
    return false;
  }

  Tree(int cap_, int size_) : cap(cap_), size(size_), cells(size_ * size_), actions(size_ * size_) {
    ko.assign(cap, -1); passes.assign(cap, 0);
    N.assign(cap, 0); VL.assign(cap, 0); parent.assign(cap, -2); action.assign(cap, -1);
    child_start.assign(cap, 0); child_count.assign(cap, 0); mc.assign(cap, 0);
    W.assign(cap, 0.f); P.assign(cap, 0.f); terminal.assign(cap, 0);
    player.assign(cap, 0); boards.assign((size_t)cap * cells, 0);
  }

  const int8_t* board(int n) const { return &boards[(size_t)n * cells]; }

  // Occurrences of node n's position: itself, its ancestors, and the positions before the root
  // (the repetition key is the piece placement, chess_rules.h).
  int chess_reps(int n, const oracle_chess_pos& p) const {
    int r = 1;
    for (int a = parent[n]; a >= 0; a = parent[a]) r += oracle_chess_same(&cpos[a], &p);
    for (const auto& q : prior) r += oracle_chess_same(&q, &p);
    return r;
  }

  void features(int n, float* out) const {
    if (game == 2) {
      const oracle_chess_pos* hist[8];
      int cur = n, k = 0;
      for (; k < 8 && cur >= 0; ++k, cur = parent[cur]) hist[k] = &cpos[cur];
      for (size_t j = 0; k < 8; ++k, ++j) hist[k] = j < prior.size() ? &prior[j] : nullptr;
      oracle_chess_features(hist, out);
      return;
    }
    if (game == 1) {
      const int8_t* hist[8];
      int cur = n, k = 0;
      for (; k < 8 && cur >= 0; ++k, cur = parent[cur]) hist[k] = board(cur);
      for (int j = 1; k < 8; ++k, ++j) hist[k] = &root_hist[(size_t)j * cells];
      oracle::go_features(hist, cells, player[n], out);
      return;
    }
    oracle::gomoku_features(board(n), size, player[n], mc[n], n == 0 ? -1 : action[n], out);
  }

  // evaluator call on a list of nodes (one evaluate_batch call)
  void evaluate(const std::vector<int>& nodes) {
    const int n = (int)nodes.size();
    if (n == 0) return;
    feat.assign((size_t)n * planes * cells, 0.f);
    pol.assign((size_t)n * actions, 0.f);
    val.assign(n, 0.f);
    for (int i = 0; i < n; ++i) features(nodes[i], &feat[(size_t)i * planes * cells]);
    if (eval)
      eval(ctx, n, feat.data(), pol.data(), val.data());
    else if (game == 1)
      oracle_synth_eval_go(n, cells, actions, feat.data(), pol.data(), val.data());
    else if (game == 2)
      oracle_synth_eval_chess(n, feat.data(), pol.data(), val.data());
    else
      oracle_synth_eval(n, oracle::kPlanes, cells, actions, feat.data(), pol.data(), val.data());
    res.eval_calls++;
    res.eval_positions += n;
  }

  float vl_value() const { return -std::fabs(cfg.virtual_loss); }
  int vl_count(int c) const { return cfg.enable_virtual_loss ? VL[c] : 0; }

  // UCB score of child c under parent visit count np (wave_search.py:1287-1296, 1059-1072;
  // node_data_manager.py:379-390).
  float score(int c, int32_t np) const {
    float ne = (float)(N[c] + vl_count(c));
    float we = W[c];
    if (cfg.enable_virtual_loss) we = W[c] + (float)VL[c] * vl_value();
    float q = ne > 0.0f ? we / ne : 0.0f;
    float sq = std::sqrt(std::max((float)np, 1.0f));
    float u = ((cfg.c_puct * P[c]) * sq) / (1.0f + ne);
    return q + u;
  }

  void add_vl(int c) { if (cfg.enable_virtual_loss) VL[c] += 1; }

  // wave_search.py:779-979 + csr_tree.py:391-449 for the unique, ascending `leaves`.
  int expand(const std::vector<int>& leaves) {
    std::vector<int> todo;
    for (int n : leaves)
      if (n >= 0 && n < num_nodes && child_count[n] == 0 && !terminal[n]) todo.push_back(n);
    if (todo.empty()) return 0;
    evaluate(todo);
    std::vector<float> pol_copy = pol;
    for (size_t i = 0; i < todo.size(); ++i) {
      const int n = todo[i];
      const float* p = &pol_copy[i * actions];
      const int8_t* b = board(n);
      std::vector<int> legal;
      std::vector<int32_t> chess_moves;  // by action, for game == 2
      if (game == 2) {
        // terminal positions are discovered when first expanded (ChessState::isTerminal order)
        int res = 0;
        if (oracle_chess_terminal(&cpos[n], cpos[n].reps, &res)) { terminal[n] = 1; continue; }
        int32_t mv[320];
        const int k = oracle_chess_legal(&cpos[n], mv);
        std::vector<std::pair<int, int32_t>> am;
        for (int j = 0; j < k; ++j) am.push_back({oracle_chess_action(&cpos[n], mv[j]), mv[j]});
        std::sort(am.begin(), am.end());
        for (auto& x : am) { legal.push_back(x.first); chess_moves.push_back(x.second); }
      } else if (game == 1) {
        std::vector<uint8_t> m(actions);
        if (superko) {
          // keys of the game so far: before the root, then every non-pass position on the path
          std::vector<uint64_t> h(root_keys);
          for (int a = n; a > 0; a = parent[a])
            if (action[a] != cells) h.push_back(node_key[a]);
          oracle::go_legal_superko(b, size, player[n], ko[n], h.data(), (int)h.size(), m.data());
        } else {
          oracle::go_legal(b, size, player[n], ko[n], m.data());
        }
        for (int a = 0; a < actions; ++a)
          if (m[a]) legal.push_back(a);
      } else {
        for (int a = 0; a < actions; ++a)
          if (b[a] == 0) legal.push_back(a);
      }
      if (legal.empty()) continue;
      // priors = p[legal] / (sum(p[legal]) + 1e-8) (wave_search.py:894-895), the sum in the order
      // torch's CPU kernel adds the gathered fp32 vector (torch_sum.cpp)
      std::vector<float> pl(legal.size());
      for (size_t j = 0; j < legal.size(); ++j) pl[j] = p[legal[j]];
      const float denom = torch_cpu_sum(pl.data(), (int)pl.size()) + 1e-8f;
      const int k = (int)legal.size();
      if (num_nodes + k > cap) return 1;  // "Tree full" (csr_tree.py:405-406)
      child_start[n] = num_nodes;
      child_count[n] = k;
      for (int j = 0; j < k; ++j) {
        const int c = num_nodes++;
        const int a = legal[j];
        N[c] = 0; W[c] = 0.f; VL[c] = 0; P[c] = p[a] / denom;
        parent[c] = n; action[c] = a; child_count[c] = 0;
        player[c] = (int8_t)(3 - player[n]);
        mc[c] = mc[n] + 1;
        if (game == 1 && cycle) {
          // Japanese / Korean repetition rule (go_state.cpp:342-356): the child's position
          // (board, ko point, side to move) occurring for the third time ends the game
          int k2 = -1;
          oracle::go_play(b, size, player[n], a, ko[n], &boards[(size_t)c * cells], &k2);
          const uint64_t key = oracle::go_key(&boards[(size_t)c * cells], size, k2) ^
                               oracle::mix64(0x3C6EF372FE94F82Bull ^ (uint64_t)(3 - player[n]));
          node_key[c] = key;
          int count = 0;
          for (uint64_t rk : root_keys) count += rk == key;
          for (int p2 = n; p2 > 0; p2 = parent[p2]) count += node_key[p2] == key;
          ko[c] = k2;
          passes[c] = a == cells ? passes[n] + 1 : 0;
          terminal[c] = (passes[c] >= 2 || count >= 2) ? 1 : 0;
          continue;
        }
        if (game == 2) {
          oracle_chess_pos q = cpos[n];
          oracle_chess_play(&q, chess_moves[j]);
          cpos[c] = q;
          cpos[c].reps = (int8_t)chess_reps(c, q);
          terminal[c] = 0;
          continue;
        }
        if (game == 1) {
          int k2 = -1;
          oracle::go_play(b, size, player[n], a, ko[n], &boards[(size_t)c * cells], &k2);
          ko[c] = k2;
          if (superko) node_key[c] = oracle::go_key(&boards[(size_t)c * cells], size, k2);
          passes[c] = a == cells ? passes[n] + 1 : 0;
          terminal[c] = passes[c] >= 2 ? 1 : 0;  // GoState::isTerminal (go_state.cpp:502-506)
          continue;
        }
        std::memcpy(&boards[(size_t)c * cells], b, cells);
        boards[(size_t)c * cells + a] = player[n];
        terminal[c] = oracle::gomoku_terminal(board(c), size) ? 1 : 0;
      }
    }
    return 0;
  }

  // Go root: hist[8][cells] (hist[0] = the root position, hist[k] = k plies earlier, zeros where
  // the game had not started), side to move, ko point (-1 none), consecutive passes.
  int begin_go(const oracle_config* c, const int8_t* hist, int to_move, int root_ko,
               int root_passes, oracle_eval_fn e, void* x, const uint64_t* keys = nullptr,
               int nkeys = 0, int sk = 0, int cy = 0) {
    game = 1;
    superko = sk;
    cycle = cy;
    root_keys.assign(keys, keys + (keys && nkeys > 0 ? nkeys : 0));
    if ((superko || cycle) && !(kept == 2 && node_key.size() == (size_t)cap)) node_key.assign(cap, 0);
    planes = oracle::kGoPlanes;
    actions = cells + 1;
    root_hist.assign(hist, hist + (size_t)8 * cells);
    cfg = *c;
    if (cfg.board_size != size || cfg.max_nodes > cap || cfg.max_wave_size <= 0) return 2;
    eval = e; ctx = x;
    res = oracle_result{};
    if (install_root()) return 0;
    std::memcpy(boards.data(), hist, cells);
    player[0] = (int8_t)to_move;
    ko[0] = root_ko;
    passes[0] = root_passes;
    mc[0] = 0;
    terminal[0] = root_passes >= 2 ? 1 : 0;
    int st = expand({0});
    res.status = st;
    return st;
  }

  // Chess root: its record (reps = occurrences in the game so far, itself included) and the
  // game's earlier positions, most recent first.
  int begin_chess(const oracle_config* c, const oracle_chess_pos* root, const oracle_chess_pos* pr,
                  int nprior, oracle_eval_fn e, void* x) {
    game = 2;
    planes = oracle::kChessPlanes;
    actions = oracle::kChessActions;
    cfg = *c;
    if (cfg.board_size != 8 || size != 8 || cfg.max_nodes > cap || cfg.max_wave_size <= 0) return 2;
    if (!(kept == 2 && cpos.size() == (size_t)cap)) cpos.assign(cap, oracle_chess_pos{});
    prior.assign(pr, pr + (nprior > 0 ? nprior : 0));
    eval = e; ctx = x;
    res = oracle_result{};
    if (install_root()) return 0;
    terminal[0] = 0;
    cpos[0] = *root;
    player[0] = root->side;
    mc[0] = 0;
    int st = expand({0});
    res.status = st;
    return st;
  }

  int begin(const oracle_config* c, const int8_t* root, oracle_eval_fn e, void* x) {
    game = 0;
    planes = oracle::kPlanes;
    actions = cells;
    cfg = *c;
    if (cfg.board_size != size || cfg.max_nodes > cap || cfg.max_wave_size <= 0) return 2;
    eval = e; ctx = x;
    res = oracle_result{};
    if (install_root()) return 0;
    terminal[0] = 0;
    int stones = 0;
    for (int i = 0; i < cells; ++i) { boards[i] = root[i]; stones += root[i] != 0; }
    player[0] = (stones % 2 == 0) ? 1 : 2;
    mc[0] = stones;
    int st = expand({0});
    res.status = st;
    return st;
  }

  int wave(int w) {
    const int D = cfg.max_depth;
    std::vector<int> path((size_t)w * D, 0), len(w, 1), cur(w, 0);
    std::vector<char> active(w, 1);
    // --- selection (wave_search.py:711-777, 1104-1335)
    for (int depth = 1; depth < D; ++depth) {
      std::map<int, std::vector<int>> groups;  // parent -> sims (ascending)
      for (int s = 0; s < w; ++s)
        if (active[s]) groups[cur[s]].push_back(s);
      if (groups.empty()) break;
      for (auto& g : groups) {
        const int p = g.first;
        const std::vector<int>& sims = g.second;
        std::vector<int> kids;
        for (int j = 0; j < child_count[p]; ++j) {
          int c = child_start[p] + j;
          if (game == 0 && p > 0 && board(p)[action[c]] != 0) continue;  // legal filter (no-op in Gomoku)
          kids.push_back(c);
        }
        if (kids.empty()) {
          for (int s : sims) active[s] = 0;
          continue;
        }
        const int n = (int)kids.size(), k = (int)sims.size();
        std::vector<float> sc(n);
        for (int i = 0; i < n; ++i) sc[i] = score(kids[i], N[p]);
        if (p == 0 && !root_noise.empty()) {  // (1 - eps) * valid_priors + eps * noise
          for (int i = 0; i < n; ++i) {
            const int c = kids[i];
            const float saved = P[c];
            P[c] = noise_keep * P[c] + noise_eps * root_noise[action[c]];
            sc[i] = score(c, N[p]);
            P[c] = saved;
          }
        }
        std::vector<int> order(n);
        for (int i = 0; i < n; ++i) order[i] = i;
        std::stable_sort(order.begin(), order.end(),
                         [&](int a, int b) { return sc[a] > sc[b]; });
        std::vector<int> sel(k);
        int used;  // number of leading ranks that receive simulations
        int boundary;
        if (k <= n) {
          for (int i = 0; i < k; ++i) sel[i] = kids[order[i]];
          used = k; boundary = k;
        } else {
          const int base = k / n, extra = k % n;
          int idx = 0;
          for (int i = 0; i < n; ++i) {
            int cnt = base + (i < extra ? 1 : 0);
            for (int t = 0; t < cnt; ++t) sel[idx++] = kids[order[i]];
          }
          used = n; boundary = extra;
        }
        if (boundary > 0 && boundary < n && sc[order[boundary - 1]] == sc[order[boundary]])
          res.boundary_ties++;
        for (int i = 1; i < used; ++i)
          if (sc[order[i - 1]] == sc[order[i]]) res.order_ties++;
        for (int i = 0; i < k; ++i) add_vl(sel[i]);
        for (int i = 0; i < k; ++i) {
          const int s = sims[i];
          path[(size_t)s * D + depth] = sel[i];
          len[s] = depth + 1;
          cur[s] = sel[i];
        }
      }
    }
    std::vector<int> leaf(w);
    for (int s = 0; s < w; ++s) leaf[s] = path[(size_t)s * D + len[s] - 1];
    // --- expansion (wave_search.py:779-979)
    std::vector<int> uniq(leaf);
    std::sort(uniq.begin(), uniq.end());
    uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
    if (expand(uniq)) { res.status = 1; return 1; }
    // --- child pick (wave_search.py:981-1102)
    std::vector<int> fin(leaf);
    for (int n : uniq) {
      if (child_count[n] == 0) continue;
      int best = -1;
      float bs = 0.f;
      for (int j = 0; j < child_count[n]; ++j) {
        int c = child_start[n] + j;
        if (game == 0 && board(n)[action[c]] != 0) continue;
        float s = score(c, N[n]);
        if (best < 0 || s > bs) { best = c; bs = s; }
      }
      if (best < 0) continue;
      add_vl(best);  // one non-accumulating += for all simulations at n
      for (int s = 0; s < w; ++s)
        if (leaf[s] == n) {
          fin[s] = best;
          if (len[s] < D) { path[(size_t)s * D + len[s]] = best; len[s] += 1; }
        }
    }
    // --- evaluation (wave_search.py:1337-1457): every simulation, duplicates included
    evaluate(fin);
    std::vector<float> v(val);
    // --- backup (mcts_gpu_accelerator.py:378-393), sequential fp32
    for (int s = 0; s < w; ++s)
      for (int d = 0; d < len[s]; ++d) {
        int n = path[(size_t)s * D + d];
        N[n] += 1;
        W[n] += (d % 2 == 0) ? v[s] : -v[s];
      }
    // --- virtual-loss revert (wave_search.py:1513-1552)
    if (cfg.enable_virtual_loss)
      for (int s = 0; s < w; ++s)
        for (int d = 1; d < len[s]; ++d) {
          int n = path[(size_t)s * D + d];
          VL[n] = std::max(VL[n] - 1, 0);
        }
    res.waves++;
    root_noise.clear();
    return 0;
  }
};

}  // namespace

extern "C" {

void* oracle_tree_create(int max_nodes, int board_size) {
  if (max_nodes < 1 || board_size < 5 || board_size > 19) return nullptr;
  return new Tree(max_nodes, board_size);
}

void oracle_tree_destroy(void* t) { delete static_cast<Tree*>(t); }

int oracle_begin(void* t, const oracle_config* cfg, const int8_t* root, oracle_eval_fn e, void* x) {
  return static_cast<Tree*>(t)->begin(cfg, root, e, x);
}

int oracle_set_root_noise(void* t, float eps, float keep, const float* noise) {
  Tree* tr = static_cast<Tree*>(t);
  tr->noise_eps = eps;
  tr->noise_keep = keep;
  tr->root_noise.assign(noise, noise + tr->actions);
  return 0;
}

int oracle_wave(void* t, int w) {
  Tree* tr = static_cast<Tree*>(t);
  if (w <= 0) return 2;
  return tr->wave(w);
}

void oracle_get_result(void* t, oracle_result* out) {
  Tree* tr = static_cast<Tree*>(t);
  *out = tr->res;
  out->num_nodes = tr->num_nodes;
}

int oracle_begin_chess(void* t, const oracle_config* cfg, const oracle_chess_pos* root,
                       const oracle_chess_pos* prior, int nprior, oracle_eval_fn e, void* x) {
  return static_cast<Tree*>(t)->begin_chess(cfg, root, prior, nprior, e, x);
}

int oracle_begin_go(void* t, const oracle_config* cfg, const int8_t* hist, int to_move, int ko,
                    int passes, oracle_eval_fn e, void* x) {
  return static_cast<Tree*>(t)->begin_go(cfg, hist, to_move, ko, passes, e, x);
}

static int run_waves(Tree* tr, const oracle_config* cfg, int st, void* t, oracle_result* out);

int oracle_begin_go_sk(void* t, const oracle_config* cfg, const int8_t* hist, int to_move, int ko,
                       int passes, const uint64_t* keys, int nkeys, int superko, oracle_eval_fn e,
                       void* x) {
  return static_cast<Tree*>(t)->begin_go(cfg, hist, to_move, ko, passes, e, x, keys, nkeys, superko);
}

int oracle_begin_go_rules(void* t, const oracle_config* cfg, const int8_t* hist, int to_move, int ko,
                          int passes, const uint64_t* keys, int nkeys, int superko, int cycle,
                          oracle_eval_fn e, void* x) {
  return static_cast<Tree*>(t)->begin_go(cfg, hist, to_move, ko, passes, e, x, keys, nkeys, superko,
                                         cycle);
}

int oracle_search_go(void* t, const oracle_config* cfg, const int8_t* hist, int to_move, int ko,
                     int passes, oracle_eval_fn e, void* x, oracle_result* out) {
  Tree* tr = static_cast<Tree*>(t);
  return run_waves(tr, cfg, tr->begin_go(cfg, hist, to_move, ko, passes, e, x), t, out);
}

int oracle_search(void* t, const oracle_config* cfg, const int8_t* root, oracle_eval_fn e,
                  void* x, oracle_result* out) {
  Tree* tr = static_cast<Tree*>(t);
  return run_waves(tr, cfg, tr->begin(cfg, root, e, x), t, out);
}

static int run_waves(Tree* tr, const oracle_config* cfg, int st, void* t, oracle_result* out) {
  int done = 0;
  while (st == 0 && done < cfg->num_simulations) {
    int w = std::min(cfg->max_wave_size, cfg->num_simulations - done);
    st = tr->wave(w);
    done += w;
  }
  tr->res.status = st;
  if (out) oracle_get_result(t, out);
  return st;
}

int oracle_export(void* t, int32_t* visits, float* wsum, float* priors, int32_t* vl,
                  int32_t* parent, int32_t* action, uint8_t* terminal) {
  Tree* tr = static_cast<Tree*>(t);
  const size_t n = tr->num_nodes;
  if (visits) std::memcpy(visits, tr->N.data(), n * 4);
  if (wsum) std::memcpy(wsum, tr->W.data(), n * 4);
  if (priors) std::memcpy(priors, tr->P.data(), n * 4);
  if (vl) std::memcpy(vl, tr->VL.data(), n * 4);
  if (parent) std::memcpy(parent, tr->parent.data(), n * 4);
  if (action) std::memcpy(action, tr->action.data(), n * 4);
  if (terminal) std::memcpy(terminal, tr->terminal.data(), n);
  return (int)n;
}

int oracle_actions(void* t) { return static_cast<Tree*>(t)->actions; }
int oracle_reroot(void* t, int action, int mode) { return static_cast<Tree*>(t)->reroot(action, mode); }

int oracle_root_policy(void* t, double* policy) {
  Tree* tr = static_cast<Tree*>(t);
  const int A = tr->actions;
  for (int a = 0; a < A; ++a) policy[a] = 0.0;
  long long total = 0;
  for (int j = 0; j < tr->child_count[0]; ++j) total += tr->N[tr->child_start[0] + j];
  const int n = tr->child_count[0];
  if (n == 0) {
    for (int a = 0; a < A; ++a) policy[a] = 1.0 / A;
    return 0;
  }
  for (int j = 0; j < n; ++j) {
    int c = tr->child_start[0] + j;
    policy[tr->action[c]] = total > 0 ? (double)tr->N[c] / (double)total : 1.0 / n;
  }
  return 0;
}
}

// mcts.cpp - wide-batch AlphaZero search over the GPU evaluator.
//
// The reference searches with one tree per call, or four trees in lockstep
// whose pending leaves go to the CPU evaluator four at a time
// (alphazero_search_batch4_reusing, src/az/alphazero.rs:388-521).  Here any
// number of trees run in lockstep: every round each tree descends to one leaf
// (prepare_batch_simulation, :1384-1495), all leaves of the round are
// evaluated in one GPU batch (trunk refresh of the side to move, policy
// accumulator refresh, threat logits, value head and per-move policy logits:
// cnnue_az_refresh / cnnue_az_policy_refresh / cnnue_az_evaluate), then each
// tree finalises its leaf (finalize_pending_leaf, :1497-1570) and backs the
// value up (finish_batch_simulation, :1360-1382).  Host-side leaf preparation
// and finalisation run on a pool of threads, one tree per task.
//
// The search arithmetic follows AzTree: PUCT with cpuct = init + factor *
// ln((visits + base) / base) (compute_cpuct, :1718-1739), first-play urgency
// reduced by sqrt of the visited prior mass (alphazero_fpu_value_reduction,
// :1795-1817), WDL sums flipped at every ply, ties broken by prior, forced
// replies (in check, or a single legal move) searched in the same simulation,
// best root move by visits, then Q, then prior (best_root_child, :1693-1716).
// Not restated: the rules engine's repetition / perpetual-chase adjudication
// and its rule-history features (leaves take the root's rule context), root
// Dirichlet noise (off by default in the reference), and search trace output.
//
// Move generation: pseudo-legal moves of Position (src/xiangqi/mod.rs) with
// the moves that leave the mover's general attacked (or facing the other
// general on an open file) removed.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/cnnue.h"

namespace cnnue {
int set_error(int status, const char* fmt, ...);
}

namespace {

using cnnue::set_error;

constexpr int kSq = 90;
constexpr uint32_t kNoChild = 0xffffffffu;

// ---- move generation ---------------------------------------------------------
inline int color_of(int v) { return v > 0 ? 0 : 1; }
inline int kind_of(int v) { return (v > 0 ? v : -v) - 1; }
inline bool on_board(int f, int r) { return f >= 0 && f < 9 && r >= 0 && r < 10; }
inline bool in_palace(int color, int f, int r) { return f >= 3 && f <= 5 && (color == 0 ? r >= 7 : r <= 2); }
inline bool own_half(int color, int r) { return color == 0 ? r >= 5 : r <= 4; }
inline bool is(const int8_t* b, int f, int r, int color, int kind) {
  if (!on_board(f, r)) return false;
  const int v = b[r * 9 + f];
  return v != 0 && color_of(v) == color && kind_of(v) == kind;
}

// The first square in scan order holding the general of `color` (piece code
// +1 Red, -1 Black), -1 if none: a branch-free scan from the end.
int general_square(const int8_t* b, int color) {
  const int8_t code = color == 0 ? 1 : -1;
  int g = -1;
  for (int sq = kSq - 1; sq >= 0; --sq) g = b[sq] == code ? sq : g;
  return g;
}

// Is `sq` attacked by `by` (the general attacks along an open file: the
// generals may not face each other)?
bool square_attacked(const int8_t* b, int sq, int by) {
  const int f = sq % 9, r = sq / 9;
  static const int orth[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
  for (auto& d : orth) {
    int tf = f + d[0], tr = r + d[1], seen = 0;
    while (on_board(tf, tr)) {
      const int v = b[tr * 9 + tf];
      if (v != 0) {
        const bool mine = color_of(v) == by;
        if (seen == 0) {
          if (mine && kind_of(v) == 4) return true;                   // rook
          if (mine && kind_of(v) == 0 && d[0] == 0) return true;      // facing general
          if (mine && kind_of(v) == 0 && (std::abs(tf - f) + std::abs(tr - r)) == 1 && in_palace(by, f, r))
            return true;                                              // general step
        } else {
          if (mine && kind_of(v) == 5) return true;                   // cannon over one screen
          break;
        }
        ++seen;
      }
      tf += d[0];
      tr += d[1];
    }
  }
  // horses: a horse at sq + (dx, dy) reaches sq if its leg is empty
  static const int hs[8][2] = {{1, 2}, {-1, 2}, {1, -2}, {-1, -2}, {2, 1}, {-2, 1}, {2, -1}, {-2, -1}};
  for (auto& h : hs) {
    const int hf = f + h[0], hr = r + h[1];
    if (!is(b, hf, hr, by, 3)) continue;
    const int lf = std::abs(h[1]) == 2 ? hf : f + h[0] / 2;
    const int lr = std::abs(h[1]) == 2 ? r + h[1] / 2 : hr;
    if (b[lr * 9 + lf] == 0) return true;
  }
  // soldiers
  const int back = by == 0 ? 1 : -1;  // a soldier of `by` one rank behind sq moves onto it
  if (is(b, f, r + back, by, 6)) return true;
  if (!own_half(by, r) && (is(b, f - 1, r, by, 6) || is(b, f + 1, r, by, 6))) return true;
  // advisors and elephants (only inside their own palace / half)
  if (in_palace(by, f, r)) {
    static const int d4[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
    for (auto& d : d4)
      if (is(b, f + d[0], r + d[1], by, 1)) return true;
  }
  if (own_half(by, r)) {
    static const int e4[4][2] = {{2, 2}, {2, -2}, {-2, 2}, {-2, -2}};
    for (auto& e : e4)
      if (is(b, f + e[0], r + e[1], by, 2) && b[(r + e[1] / 2) * 9 + f + e[0] / 2] == 0) return true;
  }
  return false;
}

struct Move {
  uint8_t from, to;
};

void pseudo_moves(const int8_t* b, int side, std::vector<Move>& out) {
  out.clear();
  for (int sq = 0; sq < kSq; ++sq) {
    const int v = b[sq];
    if (v == 0 || color_of(v) != side) continue;
    const int f = sq % 9, r = sq / 9;
    // push_if_valid_target (src/xiangqi/mod.rs:1482-1499): no own piece and
    // never a general on the target square
    auto add = [&](int tf, int tr) {
      if (!on_board(tf, tr)) return;
      const int t = b[tr * 9 + tf];
      if (t != 0 && (color_of(t) == side || kind_of(t) == 0)) return;
      out.push_back({(uint8_t)sq, (uint8_t)(tr * 9 + tf)});
    };
    switch (kind_of(v)) {
      case 0: {
        static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
        for (auto& d : o)
          if (in_palace(side, f + d[0], r + d[1])) add(f + d[0], r + d[1]);
        break;
      }
      case 1: {
        static const int d4[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
        for (auto& d : d4)
          if (in_palace(side, f + d[0], r + d[1])) add(f + d[0], r + d[1]);
        break;
      }
      case 2: {
        static const int e4[4][2] = {{2, 2}, {2, -2}, {-2, 2}, {-2, -2}};
        for (auto& e : e4) {
          const int tf = f + e[0], tr = r + e[1];
          if (on_board(tf, tr) && own_half(side, tr) && b[(r + e[1] / 2) * 9 + f + e[0] / 2] == 0) add(tf, tr);
        }
        break;
      }
      case 3: {
        static const int hs[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                                     {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
        for (auto& h : hs)
          if (on_board(f + h[2], r + h[3]) && b[(r + h[1]) * 9 + f + h[0]] == 0) add(f + h[2], r + h[3]);
        break;
      }
      case 4:
      case 5: {
        static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
        const bool cannon = kind_of(v) == 5;
        for (auto& d : o) {
          int tf = f + d[0], tr = r + d[1];
          bool screen = false;
          while (on_board(tf, tr)) {
            const int t = b[tr * 9 + tf];
            if (!cannon) {
              add(tf, tr);
              if (t != 0) break;
            } else if (!screen) {
              if (t == 0) add(tf, tr);
              else screen = true;
            } else if (t != 0) {
              add(tf, tr);
              break;
            }
            tf += d[0];
            tr += d[1];
          }
        }
        break;
      }
      default: {
        const int fwd = side == 0 ? -1 : 1;
        add(f, r + fwd);
        if (!own_half(side, r)) {
          add(f - 1, r);
          add(f + 1, r);
        }
      }
    }
  }
}

// Pieces of `by` giving check to the general on `g` (checkers_to).
int count_checkers(const int8_t* b, int g, int by) {
  const int f = g % 9, r = g / 9;
  int n = 0;
  static const int orth[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
  for (auto& d : orth) {
    int tf = f + d[0], tr = r + d[1], seen = 0;
    while (on_board(tf, tr)) {
      const int v = b[tr * 9 + tf];
      if (v != 0) {
        const bool mine = color_of(v) == by;
        if (seen == 0 && mine && (kind_of(v) == 4 || (kind_of(v) == 0 && d[0] == 0))) ++n;
        if (seen == 1) {
          if (mine && kind_of(v) == 5) ++n;
          break;
        }
        ++seen;
      }
      tf += d[0];
      tr += d[1];
    }
  }
  static const int hs[8][2] = {{1, 2}, {-1, 2}, {1, -2}, {-1, -2}, {2, 1}, {-2, 1}, {2, -1}, {-2, -1}};
  for (auto& h : hs) {
    const int hf = f + h[0], hr = r + h[1];
    if (!is(b, hf, hr, by, 3)) continue;
    const int lf = std::abs(h[1]) == 2 ? hf : f + h[0] / 2;
    const int lr = std::abs(h[1]) == 2 ? r + h[1] / 2 : hr;
    if (b[lr * 9 + lf] == 0) ++n;
  }
  const int back = by == 0 ? 1 : -1;
  n += is(b, f, r + back, by, 6);
  if (!own_half(by, r)) n += is(b, f - 1, r, by, 6) + is(b, f + 1, r, by, 6);
  return n;
}

// Legal moves: pseudo-legal moves after which the mover's general is not
// attacked (generals facing included); without a general every move stands.
// Order of Position::legal_moves (src/xiangqi/mod.rs:576-579, :1113-1131,
// :1259-1305): pieces in square order, each piece's steps in the reference's
// step tables; in check by a single piece the general's moves come first.
//
// The attack test runs on the board with the move made in place (and then
// unmade).  When the side is not in check, a move by another piece can only
// create an attack on its general (1) along a rank or file through the
// general that the move leaves or enters (rook, facing general, cannon
// screen) or (2) by leaving one of the general's four diagonal neighbours
// (the leg of a horse or the eye of an elephant aimed at it): soldiers and
// advisors need no open path, and the move removes no blocker elsewhere.
// Moves of neither kind are legal without a test; moves of kind (1) only
// rescan the one or two rays they touch (ray_attacked, the same rule as
// square_attacked's orthogonal part), kind (2) and the general's own moves
// take the full test.

// Is the general on `g` attacked along direction d by `by`, on the board with
// `moving` moved from `from` to `to`?
bool ray_attacked(const int8_t* b, int g, int df, int dr, int from, int to, int moving, int by) {
  const int f = g % 9, r = g / 9;
  int tf = f + df, tr = r + dr, seen = 0;
  while (on_board(tf, tr)) {
    const int sq = tr * 9 + tf;
    const int v = sq == from ? 0 : (sq == to ? moving : (int)b[sq]);
    if (v != 0) {
      const bool mine = color_of(v) == by;
      if (seen == 0) {
        if (mine && kind_of(v) == 4) return true;                   // rook
        if (mine && kind_of(v) == 0 && df == 0) return true;        // facing general
        if (mine && kind_of(v) == 0 && (std::abs(tf - f) + std::abs(tr - r)) == 1 && in_palace(by, f, r))
          return true;                                              // general step
      } else {
        return mine && kind_of(v) == 5;                             // cannon over one screen
      }
      ++seen;
    }
    tf += df;
    tr += dr;
  }
  return false;
}

// The direction from the general on `g` to `sq` when `sq` lies on its rank
// or file (0 none).
inline int ray_of(int g, int sq, int* df, int* dr) {
  const int gf = g % 9, gr = g / 9, f = sq % 9, r = sq / 9;
  if (f == gf && r != gr) {
    *df = 0;
    *dr = r > gr ? 1 : -1;
    return 1;
  }
  if (r == gr && f != gf) {
    *df = f > gf ? 1 : -1;
    *dr = 0;
    return 1;
  }
  return 0;
}

void legal_moves(const int8_t* b, int side, std::vector<Move>& pseudo, std::vector<Move>& out) {
  pseudo_moves(b, side, pseudo);
  const int king = general_square(b, side);
  const bool check = king >= 0 && square_attacked(b, king, 1 - side);
  if (check && count_checkers(b, king, 1 - side) == 1)
    std::stable_partition(pseudo.begin(), pseudo.end(), [&](const Move& m) { return m.from == king; });
  out.clear();
  if (king < 0) {
    out = pseudo;
    return;
  }
  const int kf = king % 9, kr = king / 9;
  auto leg = [&](int sq) { return std::abs(sq % 9 - kf) == 1 && std::abs(sq / 9 - kr) == 1; };
  int8_t c[kSq];
  std::memcpy(c, b, kSq);
  for (const Move& m : pseudo) {
    if (!check && m.from != king && !leg(m.from)) {
      int df0, dr0, df1, dr1;
      const int on0 = ray_of(king, m.from, &df0, &dr0), on1 = ray_of(king, m.to, &df1, &dr1);
      const int moving = b[m.from];
      const bool hit = (on0 && ray_attacked(b, king, df0, dr0, m.from, m.to, moving, 1 - side)) ||
                       (on1 && (!on0 || df1 != df0 || dr1 != dr0) &&
                        ray_attacked(b, king, df1, dr1, m.from, m.to, moving, 1 - side));
      if (!hit) out.push_back(m);
      continue;
    }
    const int8_t moving = c[m.from], captured = c[m.to];
    c[m.to] = moving;
    c[m.from] = 0;
    const int g = m.from == king ? m.to : king;
    if (!square_attacked(c, g, 1 - side)) out.push_back(m);
    c[m.from] = moving;
    c[m.to] = captured;
  }
}

bool in_check(const int8_t* b, int side) {
  const int g = general_square(b, side);
  return g >= 0 && square_attacked(b, g, 1 - side);
}

// Moves the policy can score: the canonical move (squares mirrored for Black)
// lies in the 2086-move dense space.  Legal moves outside it exist only for
// an advisor or elephant off its points, which play from the start position
// never produces (the reference's dense_move_index asserts on them); the
// search leaves them out.
const std::vector<uint16_t>& sparse_to_dense() {
  static const std::vector<uint16_t> t = [] {
    std::vector<uint16_t> v(kSq * kSq, 0xffff);
    cnnue_az_dense_moves(nullptr, v.data());
    return v;
  }();
  return t;
}

void searchable_moves(const int8_t* b, int side, std::vector<Move>& pseudo, std::vector<Move>& out) {
  legal_moves(b, side, pseudo, out);
  const auto& s2d = sparse_to_dense();
  size_t k = 0;
  for (const Move& m : out) {
    const int cf = side == 0 ? m.from : kSq - 1 - m.from, ct = side == 0 ? m.to : kSq - 1 - m.to;
    if (s2d[cf * kSq + ct] != 0xffff) out[k++] = m;
  }
  out.resize(k);
}

// ---- a small persistent thread pool ------------------------------------------
class Pool {
 public:
  explicit Pool(int n) {
    for (int i = 0; i < n; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  // fn(i) for i in [0, n), spread over the workers and the calling thread;
  // items are claimed in chunks from an atomic counter.
  void run(int64_t n, const std::function<void(int64_t)>& fn) {
    if (workers_.empty() || n < 2) {
      for (int64_t i = 0; i < n; ++i) fn(i);
      return;
    }
    const int64_t threads = (int64_t)workers_.size() + 1;
    {
      std::lock_guard<std::mutex> g(mu_);
      fn_ = &fn;
      n_ = n;
      grain_ = std::max<int64_t>(1, std::min<int64_t>(64, n / (threads * 8)));
      next_.store(0, std::memory_order_relaxed);
      busy_ = (int)workers_.size();
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> g(mu_);
    done_cv_.wait(g, [this] { return busy_ == 0; });
    fn_ = nullptr;
  }

 private:
  void work() {
    const int64_t n = n_, grain = grain_;
    for (;;) {
      const int64_t i0 = next_.fetch_add(grain, std::memory_order_relaxed);
      if (i0 >= n) return;
      const int64_t i1 = std::min(n, i0 + grain);
      for (int64_t i = i0; i < i1; ++i) (*fn_)(i);
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
      }
      work();
      {
        std::lock_guard<std::mutex> g(mu_);
        --busy_;
      }
      done_cv_.notify_all();
    }
  }
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int64_t)>* fn_ = nullptr;
  int64_t n_ = 0, grain_ = 1;
  std::atomic<int64_t> next_{0};
  int busy_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

// ---- the tree ------------------------------------------------------------------
struct Node {
  int8_t board[kSq];
  uint8_t side;
  bool expanded = false;
  uint32_t parent = kNoChild;
  uint32_t child_off = 0;
  uint16_t n_children = 0;
  uint32_t visits = 0;
  float wdl_sum[3] = {0.f, 0.f, 0.f};
  float value = 0.f;
  float value_wdl[3] = {0.f, 1.f, 0.f};
};

struct Child {
  Move mv;
  float prior;
  uint32_t visits = 0;
  float wdl_sum[3] = {0.f, 0.f, 0.f};
  uint32_t node = kNoChild;
};

struct Eval {
  float wdl[3];
  float value;
};

inline float wdl_utility(const float* wdl, float draw) {
  return std::min(std::max(wdl[0] - wdl[2] + draw * wdl[1], -1.0f), 1.0f);
}
inline float wdl_sum_utility(const float* sum, uint32_t visits, float draw) {
  if (visits == 0) return 0.f;
  const float v = (float)visits;
  const float w[3] = {sum[0] / v, sum[1] / v, sum[2] / v};
  return wdl_utility(w, draw);
}
inline Eval terminal_eval(float value) {
  Eval e;
  e.value = value;
  e.wdl[0] = value > 0.f ? 1.f : 0.f;
  e.wdl[1] = value == 0.f ? 1.f : 0.f;
  e.wdl[2] = value < 0.f ? 1.f : 0.f;
  return e;
}

// terminal_value (src/az/alphazero.rs:1848-1876) without the rules engine's
// repetition outcomes: a side without its general has lost.
bool terminal(const Node& n, float* value) {
  bool red = false, black = false;
  for (int sq = 0; sq < kSq; ++sq)
    if (n.board[sq] != 0 && kind_of(n.board[sq]) == 0) (color_of(n.board[sq]) == 0 ? red : black) = true;
  if (!red) {
    *value = n.side == 0 ? -1.f : 1.f;
    return true;
  }
  if (!black) {
    *value = n.side == 1 ? -1.f : 1.f;
    return true;
  }
  return false;
}

struct Sim {
  uint32_t node = 0;
  uint32_t depth = 0;
  std::vector<std::pair<uint32_t, uint32_t>> path;  // (parent node, child index)
};

struct Pending {
  Sim sim;
  std::vector<Move> moves;
  bool in_check = false;
  bool cutoff = false;
  bool root_expand = false;  // AzTree::expand(root): children, no visit, not a simulation
};

struct Tree {
  std::vector<Node> nodes;
  std::vector<Child> children;
  cnnue_mcts_limits lim;
  float rule[CNNUE_AZ_RULE_CONTEXT];
  uint64_t completed = 0;
  bool has_active = false, has_pending = false;
  Sim active;
  Pending pending;
  std::vector<Move> scratch_pseudo, scratch_moves;
  std::vector<uint8_t> scratch_mv;
  std::vector<float> scratch_prior;
  // leaf inputs of this round (filled when the leaf becomes pending)
  std::vector<uint32_t> items, threats, move_info;

  // A fresh tree for `root`, keeping every vector's capacity from the last
  // search (a search re-uses its trees).
  void reset(const Node& root, const cnnue_mcts_limits& limits) {
    nodes.clear();
    children.clear();
    nodes.push_back(root);
    lim = limits;
    completed = 0;
    has_active = has_pending = false;
    active.node = active.depth = 0;
    active.path.clear();
    clear_pending();
  }

  // The pending leaf's network inputs: trunk features, threat features and
  // the policy descriptors of its moves (cnnue_az_features,
  // cnnue_az_threat_features, cnnue_az_policy_moves).
  void leaf_inputs(bool threat_active) {
    const Node& leaf = nodes[pending.sim.node];
    items.resize(CNNUE_AZ_SQUARES);
    int cnt = 0;
    cnnue_az_features(leaf.board, leaf.side, items.data(), &cnt);
    items.resize(cnt);
    threats.clear();
    if (threat_active) {
      threats.resize(CNNUE_AZ_THREAT_MAX);
      int tc = 0;
      cnnue_az_threat_features(leaf.board, leaf.side, threats.data(), &tc);
      threats.resize(tc);
    }
    const size_t m = pending.moves.size();
    scratch_mv.resize(2 * m);
    for (size_t i = 0; i < m; ++i) {
      scratch_mv[2 * i] = pending.moves[i].from;
      scratch_mv[2 * i + 1] = pending.moves[i].to;
    }
    move_info.resize(2 * std::max<size_t>(m, 1));
    cnnue_az_policy_moves(leaf.board, leaf.side, scratch_mv.data(), (int)m, move_info.data());
  }

  void clear_pending() {
    pending.sim.node = pending.sim.depth = 0;
    pending.sim.path.clear();
    pending.moves.clear();
    pending.in_check = pending.cutoff = pending.root_expand = false;
  }

  uint32_t max_depth() const { return lim.max_depth > 0 ? (uint32_t)lim.max_depth : (uint32_t)lim.simulations; }

  float draw_score(uint32_t node) const { return nodes[node].side == nodes[0].side ? lim.draw_score : -lim.draw_score; }

  float cpuct(uint32_t visits, bool root) const {
    const float init = root ? lim.cpuct_at_root : lim.cpuct;
    const float factor = root ? lim.cpuct_factor_at_root : lim.cpuct_factor;
    if (factor <= 0.f) return init;
    const float base = std::max(root ? lim.cpuct_base_at_root : lim.cpuct_base, 1.0f);
    return init + factor * std::log(((float)visits + base) / base);
  }

  uint32_t select_child(uint32_t ni) const {
    const Node& n = nodes[ni];
    const Child* ch = &children[n.child_off];
    const bool root = ni == 0;
    const float draw = draw_score(ni);
    const float parent_sqrt = std::sqrt((float)std::max<uint32_t>(n.visits, 1));
    // alphazero_fpu_value_reduction (src/az/alphazero.rs:1795-1817)
    const float parent_q = n.visits > 0 ? wdl_sum_utility(n.wdl_sum, n.visits, draw) : wdl_utility(n.value_wdl, draw);
    const float reduction = root ? lim.fpu_value_at_root : lim.fpu_value;
    float fpu = parent_q;
    if (reduction > 0.f) {
      float visited = 0.f;
      for (uint32_t i = 0; i < n.n_children; ++i)
        if (ch[i].visits > 0) visited += std::max(ch[i].prior, 0.0f);
      visited = std::min(std::max(visited, 0.0f), 1.0f);
      fpu = std::min(std::max(parent_q - reduction * std::sqrt(visited), -1.0f), 1.0f);
    }
    const float c = cpuct(n.visits, root);
    int best = -1;
    float best_score = 0.f, best_prior = 0.f;
    for (uint32_t i = 0; i < n.n_children; ++i) {
      const float q = ch[i].visits > 0 ? wdl_sum_utility(ch[i].wdl_sum, ch[i].visits, draw) : fpu;
      const float u = c * ch[i].prior * parent_sqrt / (1.0f + (float)ch[i].visits);
      const float score = q + u;
      if (best < 0 || score > best_score || (score == best_score && ch[i].prior > best_prior)) {
        best = (int)i;
        best_score = score;
        best_prior = ch[i].prior;
      }
    }
    return best < 0 ? 0 : (uint32_t)best;
  }

  uint32_t ensure_child(uint32_t ni, uint32_t ci) {
    if (children[nodes[ni].child_off + ci].node != kNoChild) return children[nodes[ni].child_off + ci].node;
    const Move mv = children[nodes[ni].child_off + ci].mv;
    Node c;
    std::memcpy(c.board, nodes[ni].board, kSq);
    c.board[mv.to] = c.board[mv.from];
    c.board[mv.from] = 0;
    c.side = (uint8_t)(1 - nodes[ni].side);
    c.parent = ni;
    nodes.push_back(c);
    const uint32_t id = (uint32_t)nodes.size() - 1;
    children[nodes[ni].child_off + ci].node = id;
    return id;
  }

  void add_visit(uint32_t ni, const Eval& e) {
    nodes[ni].visits += 1;
    for (int k = 0; k < 3; ++k) nodes[ni].wdl_sum[k] += e.wdl[k];
  }

  // finish_batch_simulation (src/az/alphazero.rs:1360-1382)
  void finish(Sim& sim, Eval e) {
    add_visit(sim.node, e);
    for (auto it = sim.path.rbegin(); it != sim.path.rend(); ++it) {
      e.value = -e.value;
      std::swap(e.wdl[0], e.wdl[2]);
      Child& ch = children[nodes[it->first].child_off + it->second];
      ch.visits += 1;
      for (int k = 0; k < 3; ++k) ch.wdl_sum[k] += e.wdl[k];
      add_visit(it->first, e);
    }
    sim.path.clear();
    ++completed;
  }

  void set_value(uint32_t ni, const Eval& e) {
    nodes[ni].value = e.value;
    for (int k = 0; k < 3; ++k) nodes[ni].value_wdl[k] = e.wdl[k];
  }

  // prepare_batch_simulation (src/az/alphazero.rs:1384-1495): true = a leaf
  // is pending; false = the simulation completed without an evaluation.
  bool prepare(Sim& sim) {
    for (;;) {
      const uint32_t ni = sim.node;
      Node& n = nodes[ni];
      const bool cutoff = sim.depth >= max_depth();
      if (cutoff && n.expanded) {
        Eval e{{n.value_wdl[0], n.value_wdl[1], n.value_wdl[2]}, n.value};
        finish(sim, e);
        return false;
      }
      if (cutoff || !n.expanded) {
        float tv;
        if (terminal(n, &tv)) {
          const Eval e = terminal_eval(tv);
          set_value(ni, e);
          if (!cutoff) nodes[ni].expanded = true;
          finish(sim, e);
          return false;
        }
        searchable_moves(n.board, n.side, scratch_pseudo, scratch_moves);
        if (scratch_moves.empty()) {
          const Eval e{{0.f, 0.f, 1.f}, -1.f};
          set_value(ni, e);
          if (!cutoff) nodes[ni].expanded = true;
          finish(sim, e);
          return false;
        }
        clear_pending();
        std::swap(pending.sim, sim);
        pending.moves.assign(scratch_moves.begin(), scratch_moves.end());
        pending.in_check = !cutoff && in_check(n.board, n.side);
        pending.cutoff = cutoff;
        has_pending = true;
        return true;
      }
      if (n.n_children == 0) {
        Eval e{{n.value_wdl[0], n.value_wdl[1], n.value_wdl[2]}, n.value};
        finish(sim, e);
        return false;
      }
      const uint32_t ci = select_child(ni);
      const uint32_t child = ensure_child(ni, ci);
      sim.path.push_back({ni, ci});
      sim.node = child;
      sim.depth += 1;
    }
  }

  // AzTree::expand of the root (src/az/alphazero.rs:959-1081): a terminal or
  // move-less root gets its value and no children; otherwise its leaf is
  // queued for the first evaluation batch.
  void start_root() {
    Node& r = nodes[0];
    float tv;
    if (terminal(r, &tv)) {
      set_value(0, terminal_eval(tv));
      r.expanded = true;
      return;
    }
    searchable_moves(r.board, r.side, scratch_pseudo, scratch_moves);
    if (scratch_moves.empty()) {
      set_value(0, Eval{{0.f, 0.f, 1.f}, -1.f});
      r.expanded = true;
      return;
    }
    clear_pending();
    pending.moves.assign(scratch_moves.begin(), scratch_moves.end());
    pending.root_expand = true;
    has_pending = true;
  }

  // finalize_pending_leaf (src/az/alphazero.rs:1497-1570): returns true when
  // the simulation continues (a forced reply).
  bool finalize(Eval e, const float* logits) {
    Pending& p = pending;
    has_pending = false;
    const uint32_t ni = p.sim.node;
    const float scale = std::min(std::max(lim.value_scale, 0.0f), 1.0f);
    // scale_wdl_value (src/az/alphazero.rs:1839-1846)
    const float w0 = e.wdl[0] * scale, w1 = e.wdl[1] + (1.0f - scale) * (e.wdl[0] + e.wdl[2]), w2 = e.wdl[2] * scale;
    e.wdl[0] = w0;
    e.wdl[1] = w1;
    e.wdl[2] = w2;
    e.value *= lim.value_scale;
    set_value(ni, e);
    if (p.cutoff) {
      finish(p.sim, e);
      return false;
    }
    const bool root_expand = p.root_expand;
    // softmax_into (src/az/alphazero.rs:1878-1901) at the policy temperature
    const size_t m = p.moves.size();
    float mx = -INFINITY;
    for (size_t i = 0; i < m; ++i) mx = std::max(mx, logits[i]);
    const float inv_t = 1.0f / std::max(lim.policy_softmax_temp, 1.0e-3f);
    std::vector<float>& pri = scratch_prior;
    pri.resize(m);
    float sum = 0.f;
    for (size_t i = 0; i < m; ++i) {
      pri[i] = std::exp((logits[i] - mx) * inv_t);
      sum += pri[i];
    }
    const float inv_sum = 1.0f / std::max(sum, 1e-12f);
    nodes[ni].child_off = (uint32_t)children.size();
    for (size_t i = 0; i < m; ++i) {
      Child c;
      c.mv = p.moves[i];
      c.prior = pri[i] * inv_sum;
      children.push_back(c);
    }
    nodes[ni].n_children = (uint16_t)m;
    nodes[ni].expanded = true;
    if (root_expand) return false;
    if (m > 0 && (p.in_check || m == 1)) {
      std::swap(active, p.sim);
      const uint32_t child = ensure_child(ni, 0);
      active.path.push_back({ni, 0});
      active.node = child;
      active.depth += 1;
      has_active = true;
      return true;
    }
    finish(p.sim, e);
    return false;
  }
};

}  // namespace

struct cnnue_mcts {
  const cnnue_az_model* model = nullptr;
  int64_t hidden = 0;
  bool threat_active = false;
  Pool* pool = nullptr;
  std::vector<Tree> trees;
  struct Buf {  // device memory, grown on demand
    void* d = nullptr;
    size_t bytes = 0;
  };
  struct HostBuf {  // pinned host memory, grown on demand
    void* h = nullptr;
    size_t bytes = 0;
  };
  // One in-flight GPU batch: the trees are split in two halves whose rounds
  // alternate, so one half's selection runs while the other's leaves are on
  // the GPU.  Each slot has its own device buffers (one workspace per
  // evaluation call, so that each call's status word is read), pinned
  // staging and a completion event.
  struct Slot {
    Buf items, offsets, acc, pacc, threats, t_off, minfo, m_off, rule, wdl, q, logits, ws_trunk, ws_policy, ws_eval;
    HostBuf h_items, h_off, h_threats, h_toff, h_minfo, h_moff, h_rule, h_wdl, h_q, h_logits, h_status;
    cudaEvent_t done = nullptr;
    std::vector<uint32_t> ids;  // the trees whose leaves are in this batch
    bool in_flight = false;
  };
  Slot slot[2];
  // seconds spent in the last search: selection and leaf inputs; batch
  // assembly and launch; waiting for the GPU; finalisation and backup
  double t_select = 0, t_inputs = 0, t_gpu = 0, t_finalize = 0;
  uint64_t rounds = 0;
  ~cnnue_mcts() {
    for (Slot& sl : slot) {
      if (sl.in_flight && sl.done) cudaEventSynchronize(sl.done);
      for (Buf* b : {&sl.items, &sl.offsets, &sl.acc, &sl.pacc, &sl.threats, &sl.t_off, &sl.minfo, &sl.m_off, &sl.rule,
                     &sl.wdl, &sl.q, &sl.logits, &sl.ws_trunk, &sl.ws_policy, &sl.ws_eval})
        if (b->d) cudaFree(b->d);
      for (HostBuf* b : {&sl.h_items, &sl.h_off, &sl.h_threats, &sl.h_toff, &sl.h_minfo, &sl.h_moff, &sl.h_rule,
                         &sl.h_wdl, &sl.h_q, &sl.h_logits, &sl.h_status})
        if (b->h) cudaFreeHost(b->h);
      if (sl.done) cudaEventDestroy(sl.done);
    }
    delete pool;
  }
};

namespace {

int grow(cnnue_mcts::Buf& b, size_t bytes) {
  bytes = std::max<size_t>(bytes, 256);
  if (b.bytes >= bytes) return CNNUE_OK;
  if (b.d) cudaFree(b.d);
  b.d = nullptr;
  b.bytes = 0;
  const size_t want = bytes + bytes / 2;
  if (cudaMalloc(&b.d, want) != cudaSuccess) return set_error(CNNUE_ERR_CUDA, "cudaMalloc of %zu bytes", want);
  b.bytes = want;
  return CNNUE_OK;
}

// Pinned host memory, so that the round's copies run asynchronously.
template <class T>
int grow_host(cnnue_mcts::HostBuf& b, size_t count, T** out) {
  const size_t bytes = std::max<size_t>(count * sizeof(T), 256);
  if (b.bytes < bytes) {
    if (b.h) cudaFreeHost(b.h);
    b.h = nullptr;
    b.bytes = 0;
    const size_t want = bytes + bytes / 2;
    if (cudaHostAlloc(&b.h, want, cudaHostAllocDefault) != cudaSuccess)
      return set_error(CNNUE_ERR_CUDA, "cudaHostAlloc of %zu bytes", want);
    b.bytes = want;
  }
  *out = static_cast<T*>(b.h);
  return CNNUE_OK;
}

#define MCTS_TRY(x)                    \
  do {                                 \
    if (int st__ = (x)) return st__;   \
  } while (0)
#define MCTS_CUDA(x)                                                                        \
  do {                                                                                      \
    cudaError_t e__ = (x);                                                                  \
    if (e__ != cudaSuccess) return set_error(CNNUE_ERR_CUDA, "%s: %s", #x, cudaGetErrorString(e__)); \
  } while (0)

// Evaluates the pending leaves of trees[ids] in one GPU batch and finalises them.
inline double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// The kernel status word of a workspace (as cnnue_read_status decodes it).
int decode_status(uint32_t word) {
  if (word & CNNUE_STATUS_BAD_OFFSETS) return CNNUE_ERR_BAD_OFFSETS;
  if (word & CNNUE_STATUS_BAD_INDEX) return CNNUE_ERR_BAD_INDEX;
  if (word & CNNUE_STATUS_TIMEOUT) return CNNUE_ERR_TIMEOUT;
  return word != 0 ? CNNUE_ERR_INTERNAL : CNNUE_OK;
}

// Assembles the pending leaves of trees sl.ids into one batch (CSR arrays in
// the slot's pinned buffers) and queues its copies, the evaluation kernels,
// the copies back and the status words on `stream`, then the slot's event.
int launch_round(cnnue_mcts* s, cnnue_mcts::Slot& sl, cudaStream_t stream) {
  const std::vector<uint32_t>& ids = sl.ids;
  const int64_t n = (int64_t)ids.size();
  if (n == 0) return CNNUE_OK;
  const double t0 = now_s();
  // (each leaf's inputs were computed when it became pending)
  uint32_t *off, *toff, *moff;
  MCTS_TRY(grow_host(sl.h_off, n + 1, &off));
  MCTS_TRY(grow_host(sl.h_toff, n + 1, &toff));
  MCTS_TRY(grow_host(sl.h_moff, n + 1, &moff));
  off[0] = toff[0] = moff[0] = 0;
  for (int64_t k = 0; k < n; ++k) {
    const Tree& t = s->trees[ids[k]];
    off[k + 1] = off[k] + (uint32_t)t.items.size();
    toff[k + 1] = toff[k] + (uint32_t)t.threats.size();
    moff[k + 1] = moff[k] + (uint32_t)t.pending.moves.size();
  }
  const size_t n_items = std::max<uint32_t>(off[n], 1), n_threats = std::max<uint32_t>(toff[n], 1);
  const size_t n_minfo = 2 * (size_t)std::max<uint32_t>(moff[n], 1), n_rule = (size_t)n * CNNUE_AZ_RULE_CONTEXT;
  const size_t n_logits = std::max<uint32_t>(moff[n], 1), n_off = (size_t)n + 1;
  uint32_t *items, *threats, *minfo, *status;
  float *rule, *wdl, *q, *logits;
  MCTS_TRY(grow_host(sl.h_items, n_items, &items));
  MCTS_TRY(grow_host(sl.h_threats, n_threats, &threats));
  MCTS_TRY(grow_host(sl.h_minfo, n_minfo, &minfo));
  MCTS_TRY(grow_host(sl.h_rule, n_rule, &rule));
  MCTS_TRY(grow_host(sl.h_wdl, (size_t)n * 3, &wdl));
  MCTS_TRY(grow_host(sl.h_q, (size_t)n, &q));
  MCTS_TRY(grow_host(sl.h_logits, n_logits, &logits));
  MCTS_TRY(grow_host(sl.h_status, 3, &status));
  const int64_t chunk = 256;
  s->pool->run((n + chunk - 1) / chunk, [&](int64_t c) {
    for (int64_t k = c * chunk; k < std::min(n, (c + 1) * chunk); ++k) {
      const Tree& t = s->trees[ids[k]];
      std::copy(t.items.begin(), t.items.end(), items + off[k]);
      std::copy(t.threats.begin(), t.threats.end(), threats + toff[k]);
      std::copy(t.move_info.begin(), t.move_info.begin() + 2 * t.pending.moves.size(), minfo + 2 * moff[k]);
      std::copy(t.rule, t.rule + CNNUE_AZ_RULE_CONTEXT, rule + k * CNNUE_AZ_RULE_CONTEXT);
    }
  });
  const size_t ev_ws = cnnue_az_evaluate_workspace_bytes(s->model, n);
  MCTS_TRY(grow(sl.items, n_items * 4));
  MCTS_TRY(grow(sl.offsets, n_off * 4));
  MCTS_TRY(grow(sl.acc, (size_t)n * s->hidden * 4));
  MCTS_TRY(grow(sl.pacc, (size_t)n * 32 * 2));
  MCTS_TRY(grow(sl.threats, n_threats * 4));
  MCTS_TRY(grow(sl.t_off, n_off * 4));
  MCTS_TRY(grow(sl.minfo, n_minfo * 4));
  MCTS_TRY(grow(sl.m_off, n_off * 4));
  MCTS_TRY(grow(sl.rule, n_rule * 4));
  MCTS_TRY(grow(sl.wdl, (size_t)n * 12));
  MCTS_TRY(grow(sl.q, (size_t)n * 4));
  MCTS_TRY(grow(sl.logits, n_logits * 4));
  MCTS_TRY(grow(sl.ws_trunk, cnnue_az_workspace_bytes()));
  MCTS_TRY(grow(sl.ws_policy, cnnue_az_workspace_bytes()));
  MCTS_TRY(grow(sl.ws_eval, ev_ws));
  if (!sl.done) MCTS_CUDA(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
  MCTS_CUDA(cudaMemcpyAsync(sl.items.d, items, n_items * 4, cudaMemcpyHostToDevice, stream));
  MCTS_CUDA(cudaMemcpyAsync(sl.offsets.d, off, n_off * 4, cudaMemcpyHostToDevice, stream));
  MCTS_CUDA(cudaMemcpyAsync(sl.threats.d, threats, n_threats * 4, cudaMemcpyHostToDevice, stream));
  MCTS_CUDA(cudaMemcpyAsync(sl.t_off.d, toff, n_off * 4, cudaMemcpyHostToDevice, stream));
  MCTS_CUDA(cudaMemcpyAsync(sl.minfo.d, minfo, n_minfo * 4, cudaMemcpyHostToDevice, stream));
  MCTS_CUDA(cudaMemcpyAsync(sl.m_off.d, moff, n_off * 4, cudaMemcpyHostToDevice, stream));
  MCTS_CUDA(cudaMemcpyAsync(sl.rule.d, rule, n_rule * 4, cudaMemcpyHostToDevice, stream));
  MCTS_CUDA(cudaMemsetAsync(sl.ws_trunk.d, 0, sl.ws_trunk.bytes, stream));
  MCTS_CUDA(cudaMemsetAsync(sl.ws_policy.d, 0, sl.ws_policy.bytes, stream));
  MCTS_TRY(cnnue_az_refresh(s->model, (const uint32_t*)sl.items.d, off[n], (const uint32_t*)sl.offsets.d, n,
                            (float*)sl.acc.d, sl.ws_trunk.d, sl.ws_trunk.bytes, stream));
  MCTS_TRY(cnnue_az_policy_refresh(s->model, (const uint32_t*)sl.items.d, off[n], (const uint32_t*)sl.offsets.d, n,
                                   (int16_t*)sl.pacc.d, sl.ws_policy.d, sl.ws_policy.bytes, stream));
  MCTS_TRY(cnnue_az_evaluate(s->model, (const float*)sl.acc.d, nullptr, (const float*)sl.rule.d,
                             s->threat_active ? (const uint32_t*)sl.threats.d : nullptr, toff[n],
                             s->threat_active ? (const uint32_t*)sl.t_off.d : nullptr, (const int16_t*)sl.pacc.d,
                             (const uint32_t*)sl.minfo.d, moff[n], (const uint32_t*)sl.m_off.d, n, (float*)sl.wdl.d,
                             (float*)sl.q.d, (float*)sl.logits.d, sl.ws_eval.d, sl.ws_eval.bytes, stream));
  MCTS_CUDA(cudaMemcpyAsync(wdl, sl.wdl.d, (size_t)n * 3 * 4, cudaMemcpyDeviceToHost, stream));
  MCTS_CUDA(cudaMemcpyAsync(q, sl.q.d, (size_t)n * 4, cudaMemcpyDeviceToHost, stream));
  MCTS_CUDA(cudaMemcpyAsync(logits, sl.logits.d, n_logits * 4, cudaMemcpyDeviceToHost, stream));
  MCTS_CUDA(cudaMemcpyAsync(status, sl.ws_trunk.d, 4, cudaMemcpyDeviceToHost, stream));
  MCTS_CUDA(cudaMemcpyAsync(status + 1, sl.ws_policy.d, 4, cudaMemcpyDeviceToHost, stream));
  MCTS_CUDA(cudaMemcpyAsync(status + 2, sl.ws_eval.d, 4, cudaMemcpyDeviceToHost, stream));
  MCTS_CUDA(cudaEventRecord(sl.done, stream));
  sl.in_flight = true;
  s->t_inputs += now_s() - t0;
  s->rounds += 1;
  return CNNUE_OK;
}

// Waits for the slot's batch, checks its status words and finalises its
// leaves (priors, backup, forced replies).
int complete_round(cnnue_mcts* s, cnnue_mcts::Slot& sl) {
  if (!sl.in_flight) return CNNUE_OK;
  const double t0 = now_s();
  sl.in_flight = false;
  MCTS_CUDA(cudaEventSynchronize(sl.done));
  const uint32_t* status = static_cast<const uint32_t*>(sl.h_status.h);
  for (int k = 0; k < 3; ++k)
    if (int st = decode_status(status[k])) return set_error(st, "leaf evaluation reported bad input");
  const double t1 = now_s();
  const int64_t n = (int64_t)sl.ids.size();
  const float* wdl = static_cast<const float*>(sl.h_wdl.h);
  const float* q = static_cast<const float*>(sl.h_q.h);
  const float* logits = static_cast<const float*>(sl.h_logits.h);
  const uint32_t* moff = static_cast<const uint32_t*>(sl.h_moff.h);
  s->pool->run(n, [&](int64_t k) {
    Tree& t = s->trees[sl.ids[k]];
    Eval e{{wdl[k * 3], wdl[k * 3 + 1], wdl[k * 3 + 2]}, q[k]};
    t.finalize(e, logits + moff[k]);
  });
  s->t_gpu += t1 - t0;
  s->t_finalize += now_s() - t1;
  return CNNUE_OK;
}

}  // namespace

extern "C" {

void cnnue_mcts_default_limits(cnnue_mcts_limits* l) {
  if (!l) return;
  // AzSearchLimits::default (src/az/alphazero.rs:44-66)
  l->simulations = 10000;
  l->cpuct = l->cpuct_at_root = 1.5f;
  l->cpuct_base = l->cpuct_base_at_root = 19652.0f;
  l->cpuct_factor = l->cpuct_factor_at_root = 2.0f;
  l->max_depth = 0;
  l->fpu_value = 0.30f;
  l->fpu_value_at_root = 0.20f;
  l->policy_softmax_temp = 1.0f;
  l->draw_score = 0.0f;
  l->value_scale = 1.0f;
}

int cnnue_az_legal_moves(const int8_t* board, int side, uint8_t* moves, int capacity, int* count) {
  if (!board || !count || side < 0 || side > 1 || capacity < 0 || (capacity > 0 && !moves))
    return set_error(CNNUE_ERR_INVALID_ARG, "null board/count or bad side");
  for (int sq = 0; sq < kSq; ++sq)
    if (board[sq] < -7 || board[sq] > 7) return set_error(CNNUE_ERR_INVALID_ARG, "board[%d] = %d", sq, board[sq]);
  std::vector<Move> pseudo, legal;
  legal_moves(board, side, pseudo, legal);
  *count = (int)legal.size();
  if ((int)legal.size() > capacity) return set_error(CNNUE_ERR_WORKSPACE, "%zu moves, capacity %d", legal.size(), capacity);
  for (size_t i = 0; i < legal.size(); ++i) {
    moves[2 * i] = legal[i].from;
    moves[2 * i + 1] = legal[i].to;
  }
  return CNNUE_OK;
}

int cnnue_mcts_create(const cnnue_az_model* model, const cnnue_az_weights* weights, int n_threads, cnnue_mcts** out) {
  if (!model || !weights || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null model, weights or out");
  cnnue_mcts* s = new (std::nothrow) cnnue_mcts();
  if (!s) return set_error(CNNUE_ERR_INVALID_ARG, "out of host memory");
  s->model = model;
  s->hidden = cnnue_az_weights_hidden(weights);
  int threat = 0, tactical = 0;
  cnnue_az_quant_flags(weights, &threat, &tactical);
  s->threat_active = threat != 0;
  int t = n_threads > 0 ? n_threads : (int)std::min<unsigned>(std::max(1u, std::thread::hardware_concurrency()), 16u);
  s->pool = new Pool(t - 1);
  *out = s;
  return CNNUE_OK;
}

int cnnue_mcts_destroy(cnnue_mcts* s) {
  delete s;
  return CNNUE_OK;
}

namespace {
int search_on_device(cnnue_mcts* s, const int8_t* boards, const uint8_t* sides, const float* rule_context,
                     int64_t n_roots, const cnnue_mcts_limits* limits, void* stream, uint64_t* n_evaluations);
}

int cnnue_mcts_search(cnnue_mcts* s, const int8_t* boards, const uint8_t* sides, const float* rule_context,
                      int64_t n_roots, const cnnue_mcts_limits* limits, void* stream, uint64_t* n_evaluations) {
  if (!s || !limits || n_roots < 0 || (n_roots > 0 && (!boards || !sides)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null search, limits, boards or sides");
  if (limits->simulations < 0) return set_error(CNNUE_ERR_INVALID_ARG, "negative simulations");
  // the staging buffers and every launch go to the model's device
  int prev = -1;
  MCTS_CUDA(cudaGetDevice(&prev));
  const int dev = cnnue_az_model_device(s->model);
  if (dev != prev) MCTS_CUDA(cudaSetDevice(dev));
  const int st = search_on_device(s, boards, sides, rule_context, n_roots, limits, stream, n_evaluations);
  if (dev != prev) cudaSetDevice(prev);
  return st;
}

}  // extern "C"

namespace {
int search_on_device(cnnue_mcts* s, const int8_t* boards, const uint8_t* sides, const float* rule_context,
                     int64_t n_roots, const cnnue_mcts_limits* limits, void* stream, uint64_t* n_evaluations) {
  cudaStream_t st = (cudaStream_t)stream;
  if ((int64_t)s->trees.size() != n_roots) s->trees.resize(n_roots);
  for (int64_t i = 0; i < n_roots; ++i) {
    Tree& t = s->trees[i];
    for (int sq = 0; sq < kSq; ++sq)
      if (boards[i * kSq + sq] < -7 || boards[i * kSq + sq] > 7)
        return set_error(CNNUE_ERR_INVALID_ARG, "root %lld: board[%d] = %d", (long long)i, sq, boards[i * kSq + sq]);
    if (sides[i] > 1) return set_error(CNNUE_ERR_INVALID_ARG, "root %lld: side %d", (long long)i, sides[i]);
    Node root;
    std::memcpy(root.board, boards + i * kSq, kSq);
    root.side = sides[i];
    t.reset(root, *limits);
    for (int k = 0; k < CNNUE_AZ_RULE_CONTEXT; ++k)
      t.rule[k] = rule_context ? rule_context[i * CNNUE_AZ_RULE_CONTEXT + k] : 0.f;
  }
  uint64_t evals = 0;
  s->t_select = s->t_inputs = s->t_gpu = s->t_finalize = 0;
  s->rounds = 0;
  for (cnnue_mcts::Slot& sl : s->slot) {  // a batch left by a failed search
    if (sl.in_flight) cudaEventSynchronize(sl.done);
    sl.in_flight = false;
  }
  // every root is expanded first, in one batch (tree.expand(root), :440-445)
  {
    const double ts = now_s();
    s->pool->run(n_roots, [&](int64_t i) {
      Tree& t = s->trees[i];
      if (t.lim.simulations <= 0) return;
      t.start_root();
      if (t.has_pending) t.leaf_inputs(s->threat_active);
    });
    cnnue_mcts::Slot& sl = s->slot[0];
    sl.ids.clear();
    for (int64_t i = 0; i < n_roots; ++i)
      if (s->trees[i].has_pending) sl.ids.push_back((uint32_t)i);
    s->t_select += now_s() - ts;
    evals += sl.ids.size();
    MCTS_TRY(launch_round(s, sl, st));
    MCTS_TRY(complete_round(s, sl));
  }
  // Then rounds alternate between the two halves of the roots: finalise a
  // half's last batch, run its selection (each tree to its next leaf) and
  // launch its new batch, which the GPU runs while the other half does the
  // same.  Trees are independent, so each tree's search is the same as in
  // one batch of all roots.
  const int64_t bounds[3] = {0, n_roots / 2, n_roots};
  bool live[2] = {true, true};
  while (live[0] || live[1]) {
    for (int h = 0; h < 2; ++h) {
      if (!live[h]) continue;
      cnnue_mcts::Slot& sl = s->slot[h];
      MCTS_TRY(complete_round(s, sl));
      const double ts = now_s();
      const int64_t lo = bounds[h], hi = bounds[h + 1];
      s->pool->run(hi - lo, [&](int64_t k) {
        Tree& t = s->trees[lo + k];
        while (!t.has_pending && t.completed < (uint64_t)t.lim.simulations) {
          if (!t.has_active) {  // a new simulation from the root
            t.active.node = t.active.depth = 0;
            t.active.path.clear();
          }
          t.has_active = false;
          if (t.prepare(t.active)) {
            t.leaf_inputs(s->threat_active);
            break;
          }
        }
      });
      sl.ids.clear();
      for (int64_t i = lo; i < hi; ++i)
        if (s->trees[i].has_pending) sl.ids.push_back((uint32_t)i);
      s->t_select += now_s() - ts;
      if (sl.ids.empty()) {
        live[h] = false;
        continue;
      }
      evals += sl.ids.size();
      MCTS_TRY(launch_round(s, sl, st));
    }
  }
  if (n_evaluations) *n_evaluations = evals;
  return CNNUE_OK;
}
}  // namespace

extern "C" {

int cnnue_mcts_stats(const cnnue_mcts* s, double* seconds, uint64_t* rounds) {
  if (!s || !seconds) return set_error(CNNUE_ERR_INVALID_ARG, "null search or seconds");
  seconds[0] = s->t_select;
  seconds[1] = s->t_inputs;
  seconds[2] = s->t_gpu;
  seconds[3] = s->t_finalize;
  if (rounds) *rounds = s->rounds;
  return CNNUE_OK;
}

int cnnue_mcts_result(const cnnue_mcts* s, int64_t root, uint8_t* moves, uint32_t* visits, float* priors, float* q,
                      int capacity, int* n_moves, int* best, float* root_q, uint32_t* root_visits) {
  if (!s || root < 0 || root >= (int64_t)s->trees.size() || !n_moves)
    return set_error(CNNUE_ERR_INVALID_ARG, "bad search handle or root");
  const Tree& t = s->trees[root];
  const Node& r = t.nodes[0];
  *n_moves = r.n_children;
  const float draw = t.lim.draw_score;
  if (root_q) *root_q = wdl_sum_utility(r.wdl_sum, r.visits, draw);
  if (root_visits) *root_visits = r.visits;
  if (r.n_children > capacity) return set_error(CNNUE_ERR_WORKSPACE, "%d root moves, capacity %d", r.n_children, capacity);
  int bi = -1;
  uint32_t bv = 0;
  float bq = 0.f, bp = 0.f;
  for (uint32_t i = 0; i < r.n_children; ++i) {
    const Child& c = t.children[r.child_off + i];
    const float cq = c.visits == 0 ? 0.f : wdl_sum_utility(c.wdl_sum, c.visits, draw);
    if (moves) {
      moves[2 * i] = c.mv.from;
      moves[2 * i + 1] = c.mv.to;
    }
    if (visits) visits[i] = c.visits;
    if (priors) priors[i] = c.prior;
    if (q) q[i] = cq;
    // best_root_child (src/az/alphazero.rs:1693-1716)
    if (bi < 0 || c.visits > bv || (c.visits == bv && (cq > bq || (cq == bq && c.prior > bp)))) {
      bi = (int)i;
      bv = c.visits;
      bq = cq;
      bp = c.prior;
    }
  }
  if (best) *best = bi;
  return CNNUE_OK;
}

}  // extern "C"

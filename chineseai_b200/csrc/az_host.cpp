// az_host.cpp - host side of the reference-native AZ-NNUE evaluator.
//
// Board parsing (Position::from_fen, src/xiangqi/mod.rs:163-207), the
// side-relative feature items with their king-palace buckets (src/nnue.rs:25-43,
// src/az.rs:168-203), the items a move adds and removes
// (apply_transition_for_perspective, src/az.rs:439-566), deterministic weights
// (AzNnue::random_with_arch, src/az.rs:1339-1431) and the weight file
// (AzNnue::save / load / validate, src/az.rs:1437-1529, :2453-2499).
//
// The weight file is safetensors: an 8-byte little-endian header length, a
// JSON header {"name": {"dtype", "shape", "data_offsets"}} padded with spaces
// to a multiple of 8 bytes, then the raw little-endian tensor bytes.  Files are
// written with the tensors sorted by name, each tensor's bytes in that order.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "../../include/cnnue.h"
#include "az_weights.h"

namespace cnnue {
int set_error(int status, const char* fmt, ...);
}

namespace {

using cnnue::set_error;

constexpr int kSq = CNNUE_AZ_SQUARES;
constexpr int kDenseMoves = 2086;  // DENSE_MOVE_SPACE (src/az.rs:60, checked by :3344-3352)

// One tensor of az_weight_tensors!: rows x cols, a dimension of -1 meaning H.
struct TensorSpec {
  const char* name;
  int64_t rows;  // -1 = H; 0 = a 1-D tensor of `cols`
  int64_t cols;  // -1 = H
};

constexpr TensorSpec kSpecs[CNNUE_AZ_TENSORS] = {
    {"input_hidden", 1260, -1},
    {"input_piece_hidden", 14, -1},
    {"input_rank_hidden", 10, -1},
    {"input_file_hidden", 9, -1},
    {"input_king_piece_hidden", 252, -1},
    {"rule_context_hidden", 7, -1},
    {"hidden_bias", 0, -1},
    {"value_head_hidden", 96, -1},
    {"value_head_bias", 0, 96},
    {"value_head_output", 3, 96},
    {"value_threat_embedding", 57702, 64},
    {"value_threat_output", 3, 128},
    {"policy_threat_context", 16, 128},
    {"policy_move_bias", 0, kDenseMoves},
    {"policy_consequence_output", 0, 32},
    {"policy_context_hidden", 16, -1},
    {"policy_move_context", kDenseMoves, 16},
    {"policy_accumulator_hidden", 32, -1},
    {"policy_accumulator_move", kDenseMoves, 32},
    {"policy_sparse_table", 0, 2396815},
    {"policy_sparse_factor", 0, 199458},
    {"policy_tactical", 0, 934976},
};

inline int64_t dim(int64_t d, int64_t h) { return d < 0 ? h : d; }

std::vector<int64_t> shape_of(int i, int64_t h) {
  const TensorSpec& s = kSpecs[i];
  if (s.rows == 0) return {dim(s.cols, h)};
  return {dim(s.rows, h), dim(s.cols, h)};
}

int64_t count_of(int i, int64_t h) {
  int64_t n = 1;
  for (int64_t d : shape_of(i, h)) n *= d;
  return n;
}

// ---- SplitMix64 as the reference defines it (src/az.rs:3146-3176) ----------
struct SplitMix {
  uint64_t state;
  uint64_t next() {
    uint64_t v = state + 0x9E3779B97F4A7C15ull;
    v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
    v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
    state = v ^ (v >> 31);
    return state;
  }
  float unit_f32() { return (float)((double)(next() >> 11) * (1.0 / 9007199254740992.0)); }
  float weight(float scale) { return (unit_f32() * 2.0f - 1.0f) * scale; }
};

// ---- board helpers ---------------------------------------------------------
inline int canonical_square(int perspective, int sq) { return perspective == 0 ? sq : kSq - 1 - sq; }

// canonical_general_bucket (src/az.rs:194-203).
inline int general_bucket(int piece_index, int sq) {
  const int o = piece_index < 7 ? sq : kSq - 1 - sq;
  int file = o % 9, rank = o / 9;
  file = file < 3 ? 3 : (file > 5 ? 5 : file);
  rank = rank < 7 ? 7 : (rank > 9 ? 9 : rank);
  return (rank - 7) * 3 + (file - 3);
}

inline bool piece_ok(int v) { return v >= -7 && v <= 7; }

// Feature of the piece `v` on `sq` for `perspective` (src/nnue.rs:25-28).
inline uint32_t feature_of(int v, int sq, int perspective) {
  const int color = v > 0 ? 0 : 1, kind = (v > 0 ? v : -v) - 1;
  const int piece_index = (color == perspective ? 0 : 7) + kind;
  return (uint32_t)(piece_index * kSq + canonical_square(perspective, sq));
}

// The last square in scan order holding the general of `color` (piece code
// +1 Red, -1 Black), -1 if none: a branch-free scan.
inline int last_general(const int8_t* board, int color) {
  const int8_t code = color == 0 ? 1 : -1;
  int g = -1;
  for (int sq = 0; sq < kSq; ++sq) g = board[sq] == code ? sq : g;
  return g;
}

// (us, them) buckets of a board for a perspective: the last general of each
// side in scan order, 4 when absent (canonical_general_buckets_from_features).
void buckets_of(const int8_t* board, int perspective, int* us, int* them) {
  const int own = last_general(board, perspective), enemy = last_general(board, 1 - perspective);
  *us = own < 0 ? 4 : general_bucket(0, canonical_square(perspective, own));
  *them = enemy < 0 ? 4 : general_bucket(7, canonical_square(perspective, enemy));
}

inline uint32_t pack(uint32_t feature, int us, int them) {
  return feature | ((uint32_t)us << 11) | ((uint32_t)them << 15);
}

int check_board(const int8_t* board) {
  if (board == nullptr) return set_error(CNNUE_ERR_INVALID_ARG, "null board");
  for (int sq = 0; sq < kSq; ++sq)
    if (!piece_ok(board[sq]))
      return set_error(CNNUE_ERR_INVALID_ARG, "board[%d] = %d is not a piece code", sq, board[sq]);
  return CNNUE_OK;
}

int features(const int8_t* board, int perspective, uint32_t* items) {
  int us, them, n = 0;
  buckets_of(board, perspective, &us, &them);
  for (int sq = 0; sq < kSq; ++sq)
    if (board[sq] != 0) items[n++] = pack(feature_of(board[sq], sq, perspective), us, them);
  return n;
}

// ---- a minimal JSON reader for the safetensors header ---------------------
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  double number = 0.0;
  bool integral = false;
  int64_t integer = 0;
  std::string str;
  std::vector<Json> items;
  std::vector<std::pair<std::string, Json>> fields;
  const Json* get(const char* key) const {
    for (const auto& f : fields)
      if (f.first == key) return &f.second;
    return nullptr;
  }
};

struct JsonParser {
  const char* p;
  const char* end;
  int depth = 0;
  bool fail = false;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(end - p) < n || memcmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  bool string(std::string& out) {
    if (p >= end || *p != '"') return false;
    ++p;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return false;
        switch (*p) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u':  // kept verbatim: tensor names of this format are ASCII
            if (end - p < 5) return false;
            out.append(p - 1, 6);
            p += 4;
            break;
          default: return false;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool value(Json& v) {
    if (++depth > 64) return false;
    ws();
    if (p >= end) return false;
    bool ok = true;
    if (*p == '{') {
      v.kind = Json::Object;
      ++p;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        for (;;) {
          ws();
          std::string key;
          if (!string(key)) { ok = false; break; }
          ws();
          if (p >= end || *p != ':') { ok = false; break; }
          ++p;
          Json child;
          if (!value(child)) { ok = false; break; }
          v.fields.emplace_back(std::move(key), std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == '}') { ++p; break; }
          ok = false;
          break;
        }
      }
    } else if (*p == '[') {
      v.kind = Json::Array;
      ++p;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        for (;;) {
          Json child;
          if (!value(child)) { ok = false; break; }
          v.items.push_back(std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == ']') { ++p; break; }
          ok = false;
          break;
        }
      }
    } else if (*p == '"') {
      v.kind = Json::String;
      ok = string(v.str);
    } else if (lit("true")) {
      v.kind = Json::Bool;
      v.number = 1;
    } else if (lit("false")) {
      v.kind = Json::Bool;
    } else if (lit("null")) {
      v.kind = Json::Null;
    } else {
      const char* s = p;
      while (p < end && (strchr("+-.eE", *p) != nullptr || (*p >= '0' && *p <= '9'))) ++p;
      if (p == s) return false;
      std::string text(s, p);
      char* stop = nullptr;
      v.kind = Json::Number;
      v.number = strtod(text.c_str(), &stop);
      ok = stop != nullptr && *stop == '\0';
      v.integral = text.find_first_of(".eE") == std::string::npos;
      if (v.integral) v.integer = strtoll(text.c_str(), nullptr, 10);
    }
    --depth;
    return ok;
  }
};

struct FileCloser {
  void operator()(FILE* f) const {
    if (f) fclose(f);
  }
};
using File = std::unique_ptr<FILE, FileCloser>;

int read_file(const char* path, std::vector<char>& bytes) {
  File f(fopen(path, "rb"));
  if (!f) return set_error(CNNUE_ERR_IO, "cannot open %s for reading", path);
  if (fseek(f.get(), 0, SEEK_END) != 0) return set_error(CNNUE_ERR_IO, "cannot seek %s", path);
  const long size = ftell(f.get());
  if (size < 0 || fseek(f.get(), 0, SEEK_SET) != 0) return set_error(CNNUE_ERR_IO, "cannot size %s", path);
  try {
    bytes.resize((size_t)size);
  } catch (const std::bad_alloc&) {
    return set_error(CNNUE_ERR_IO, "out of host memory reading %s", path);
  }
  if (size > 0 && fread(bytes.data(), 1, (size_t)size, f.get()) != (size_t)size)
    return set_error(CNNUE_ERR_IO, "short read on %s", path);
  return CNNUE_OK;
}

struct TensorRef {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;
};

// Parses a safetensors file into name -> tensor; checks offsets and sizes.
int parse_safetensors(const std::vector<char>& bytes, std::map<std::string, TensorRef>& out,
                      const char** data) {
  if (bytes.size() < 8) return set_error(CNNUE_ERR_FORMAT, "safetensors file shorter than its header length");
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | (uint8_t)bytes[i];
  if (n > bytes.size() - 8) return set_error(CNNUE_ERR_FORMAT, "safetensors header length %llu past the file end",
                                             (unsigned long long)n);
  JsonParser parser{bytes.data() + 8, bytes.data() + 8 + n};
  Json root;
  if (!parser.value(root) || root.kind != Json::Object)
    return set_error(CNNUE_ERR_FORMAT, "safetensors header is not a JSON object");
  parser.ws();
  if (parser.p != parser.end) return set_error(CNNUE_ERR_FORMAT, "trailing bytes in the safetensors header");
  const uint64_t data_len = bytes.size() - 8 - n;
  *data = bytes.data() + 8 + n;
  for (const auto& f : root.fields) {
    if (f.first == "__metadata__") continue;
    const Json& t = f.second;
    const Json* dt = t.get("dtype");
    const Json* sh = t.get("shape");
    const Json* off = t.get("data_offsets");
    if (t.kind != Json::Object || !dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !off ||
        off->kind != Json::Array || off->items.size() != 2)
      return set_error(CNNUE_ERR_FORMAT, "safetensors entry `%s` is malformed", f.first.c_str());
    TensorRef r;
    r.dtype = dt->str;
    for (const Json& d : sh->items) {
      if (d.kind != Json::Number || !d.integral || d.integer < 0)
        return set_error(CNNUE_ERR_FORMAT, "tensor `%s` has a bad shape", f.first.c_str());
      r.shape.push_back(d.integer);
    }
    for (int k = 0; k < 2; ++k)
      if (off->items[k].kind != Json::Number || !off->items[k].integral || off->items[k].integer < 0)
        return set_error(CNNUE_ERR_FORMAT, "tensor `%s` has bad data_offsets", f.first.c_str());
    r.begin = (uint64_t)off->items[0].integer;
    r.end = (uint64_t)off->items[1].integer;
    if (r.begin > r.end || r.end > data_len)
      return set_error(CNNUE_ERR_FORMAT, "tensor `%s` data_offsets [%llu, %llu) outside the %llu data bytes",
                       f.first.c_str(), (unsigned long long)r.begin, (unsigned long long)r.end,
                       (unsigned long long)data_len);
    out[f.first] = std::move(r);
  }
  return CNNUE_OK;
}

// Loads one F32 tensor, flattened (load_candle_f32_tensor, src/az.rs:222-239).
int load_f32(const std::map<std::string, TensorRef>& tensors, const char* data, const char* name,
             std::vector<float>& out) {
  auto it = tensors.find(name);
  if (it == tensors.end()) return set_error(CNNUE_ERR_FORMAT, "cannot find tensor %s", name);
  const TensorRef& r = it->second;
  if (r.dtype != "F32") return set_error(CNNUE_ERR_FORMAT, "tensor `%s` is %s, expected F32", name, r.dtype.c_str());
  uint64_t n = 1;
  for (int64_t d : r.shape) n *= (uint64_t)d;
  if (r.end - r.begin != n * 4)
    return set_error(CNNUE_ERR_FORMAT, "tensor `%s`: %llu data bytes for %llu elements", name,
                     (unsigned long long)(r.end - r.begin), (unsigned long long)n);
  out.resize(n);
  if (n) memcpy(out.data(), data + r.begin, n * 4);
  return CNNUE_OK;
}

// ---- quantised tables (src/az.rs:2201-2342) --------------------------------
constexpr int kRank = CNNUE_AZ_POLICY_RANK;

// dot_product (src/az.rs:2730-2766) as it runs on x86-64 with AVX2 and FMA:
// n >= 64 uses dot_product_avx2_fma (:2880-2922), four 8-lane fused
// accumulators over 32-float chunks, combined (a0 + a1) + (a2 + a3) per lane,
// the 8 lanes summed in order, then the tail; shorter rows use four scalar
// accumulators, (s0 + s1) + (s2 + s3), then the tail.
float reference_dot(const float* l, const float* r, int64_t n) {
  if (n >= 64) {
    float acc[4][8] = {};
    const int64_t chunks = n / 32;
    for (int64_t c = 0; c < chunks; ++c)
      for (int a = 0; a < 4; ++a)
        for (int k = 0; k < 8; ++k) {
          const int64_t i = c * 32 + a * 8 + k;
          acc[a][k] = std::fma(l[i], r[i], acc[a][k]);
        }
    float sum = 0.0f;
    for (int k = 0; k < 8; ++k) sum += (acc[0][k] + acc[1][k]) + (acc[2][k] + acc[3][k]);
    for (int64_t i = chunks * 32; i < n; ++i) sum += l[i] * r[i];
    return sum;
  }
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t chunks = n / 4;
  for (int64_t c = 0; c < chunks; ++c)
    for (int k = 0; k < 4; ++k) s[k] += l[4 * c + k] * r[4 * c + k];
  float sum = (s[0] + s[1]) + (s[2] + s[3]);
  for (int64_t i = chunks * 4; i < n; ++i) sum += l[i] * r[i];
  return sum;
}

// Symmetric per-tensor int8 quantisation; returns the scale.
float quantize_i8(const float* x, size_t n, std::vector<int8_t>& q) {
  float mx = 0.f;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, std::fabs(x[i]));
  const float scale = std::fmax(mx / 127.0f, 1.0e-12f);
  q.resize(n);
  for (size_t i = 0; i < n; ++i) {
    const float v = std::round(x[i] / scale);
    q[i] = std::isnan(v) ? (int8_t)0 : (int8_t)std::fmin(std::fmax(v, -127.f), 127.f);
  }
  return scale;
}

bool advisor_point(int r, int f) {
  return ((r == 0 || r == 2 || r == 7 || r == 9) && (f == 3 || f == 5)) || ((r == 1 || r == 8) && f == 4);
}
bool elephant_point(int r, int f) {
  return ((r == 0 || r == 9 || r == 4 || r == 5) && (f == 2 || f == 6)) ||
         ((r == 2 || r == 7) && (f == 0 || f == 4 || f == 8));
}
// is_valid_policy_move (src/az.rs:3206-3237).
bool policy_move(int from, int to) {
  const int ff = from % 9, fr = from / 9, tf = to % 9, tr = to / 9;
  const int df = std::abs(tf - ff), dr = std::abs(tr - fr);
  if (df == 0 || dr == 0) return true;
  if (df + dr == 3 && df != 0 && dr != 0) return true;  // horse step
  if (df == 1 && dr == 1) return advisor_point(fr, ff) && advisor_point(tr, tf);
  if (df == 2 && dr == 2) return elephant_point(fr, ff) && elephant_point(tr, tf);
  return false;
}

const std::vector<uint16_t>& dense_moves() {
  static const std::vector<uint16_t> moves = [] {
    std::vector<uint16_t> m;
    for (int from = 0; from < kSq; ++from)
      for (int to = 0; to < kSq; ++to)
        if (from != to && policy_move(from, to)) m.push_back((uint16_t)(from * kSq + to));
    return m;
  }();
  return moves;
}

int quantize(cnnue_az_weights& w) {
  const int64_t h = w.hidden;
  const auto& moves = dense_moves();
  if ((int)moves.size() != kDenseMoves) return set_error(CNNUE_ERR_INTERNAL, "dense move space %zu", moves.size());
  // 1546 trunk rows projected on policy_accumulator_hidden.
  std::vector<float> projected;
  projected.reserve((size_t)CNNUE_AZ_POLICY_ROWS * kRank);
  const float* proj = w.t[17].data();
  for (int t : {0, 1, 2, 3, 4, 6}) {
    const std::vector<float>& table = w.t[t];
    for (size_t row = 0; row * h < table.size(); ++row)
      for (int j = 0; j < kRank; ++j) projected.push_back(reference_dot(table.data() + row * h, proj + j * h, h));
  }
  w.scale[0] = quantize_i8(projected.data(), projected.size(), w.q8[0]);
  w.scale[1] = quantize_i8(w.t[18].data(), w.t[18].size(), w.q8[1]);
  // policy_sparse_factor folded into the main part of policy_sparse_table,
  // factor order of policy_sparse_factor_indices (src/az.rs:789-813).
  std::vector<float> folded(w.t[19]);
  const int64_t move_piece = (int64_t)kDenseMoves * 14, move_king = (int64_t)kDenseMoves * 81, piece_king = 14 * 81;
  const int64_t distance_off = move_piece + move_king + piece_king, approach_off = distance_off + 14 * 6;
  const float* factor = w.t[20].data();
  for (int m = 0; m < kDenseMoves; ++m) {
    const int from = moves[m] / kSq, to = moves[m] % kSq;
    for (int piece = 0; piece < 14; ++piece)
      for (int us = 0; us < 9; ++us)
        for (int them = 0; them < 9; ++them) {
          // policy_king_distance_buckets (src/az.rs:841-859): Manhattan
          // distances from the opponent general's palace square.
          const int king = kSq - 1 - ((7 + them / 3) * 9 + 3 + them % 3);
          const int before = std::abs(from / 9 - king / 9) + std::abs(from % 9 - king % 9);
          const int after = std::abs(to / 9 - king / 9) + std::abs(to % 9 - king % 9);
          const int approach = std::min(std::max(before - after, -2), 2) + 2;
          const int distance = std::min(after, 5);
          const int pair = us * 9 + them;
          float& main = folded[(size_t)((((int64_t)m * 14 + piece) * 9 + us) * 9 + them)];
          main += factor[(int64_t)m * 14 + piece];
          main += factor[move_piece + (int64_t)m * 81 + pair];
          main += factor[move_piece + move_king + piece * 81 + pair];
          main += factor[distance_off + piece * 6 + distance];
          main += factor[approach_off + piece * 5 + approach];
        }
  }
  w.scale[2] = quantize_i8(folded.data(), folded.size(), w.q8[2]);
  // moved-piece delta and capture caches in the int8 feature and move spaces.
  w.q32[0].assign((size_t)kDenseMoves * 14, 0);
  w.q32[1].assign((size_t)kDenseMoves * 14, 0);
  const int8_t* fq = w.q8[0].data();
  const int8_t* mq = w.q8[1].data();
  for (int m = 0; m < kDenseMoves; ++m) {
    const int from = moves[m] / kSq, to = moves[m] % kSq;
    for (int piece = 0; piece < 14; ++piece) {
      int32_t delta = 0, cap = 0;
      for (int j = 0; j < kRank; ++j) {
        const int32_t wt = mq[m * kRank + j];
        const int32_t tq = fq[(piece * kSq + to) * kRank + j], fr = fq[(piece * kSq + from) * kRank + j];
        delta += (tq - fr) * wt;
        cap += tq * wt;
      }
      w.q32[0][(size_t)m * 14 + piece] = delta;
      w.q32[1][(size_t)m * 14 + piece] = cap;
    }
  }
  auto any = [](const std::vector<float>& v) {
    for (float x : v)
      if (x != 0.f) return true;
    return false;
  };
  // piece-square consequence scores over the first min(32, H) columns.
  const int64_t cs = h < 32 ? h : 32;
  w.ps_scores.resize(CNNUE_AZ_INPUT);
  for (int f = 0; f < CNNUE_AZ_INPUT; ++f) w.ps_scores[f] = reference_dot(w.t[0].data() + f * h, w.t[14].data(), cs);
  w.value_threat_active = any(w.t[11]) || any(w.t[12]);
  w.policy_tactical_active = any(w.t[21]);
  w.scale[3] = quantize_i8(w.t[10].data(), w.t[10].size(), w.q8[3]);
  return CNNUE_OK;
}

// ---- threat features (src/az.rs:577-742; src/xiangqi/mod.rs:286-389) -------
constexpr int kPieces = 14;

// threat_reachable_square (src/az.rs:663-697), canonical coordinates: own
// pieces (index < 7) live at the high ranks.
bool threat_reachable(int piece, int square) {
  const int rank = square / 9, file = square % 9;
  const bool ours = piece < 7;
  switch (piece % 7) {
    case 0: return file >= 3 && file <= 5 && (ours ? rank >= 7 : rank <= 2);
    case 1:
      return ours ? ((rank == 7 || rank == 9) && (file == 3 || file == 5)) || (rank == 8 && file == 4)
                  : ((rank == 0 || rank == 2) && (file == 3 || file == 5)) || (rank == 1 && file == 4);
    case 2:
      return ours ? (rank == 5 && (file == 2 || file == 6)) || (rank == 7 && (file == 0 || file == 4 || file == 8)) ||
                        (rank == 9 && (file == 2 || file == 6))
                  : (rank == 0 && (file == 2 || file == 6)) || (rank == 2 && (file == 0 || file == 4 || file == 8)) ||
                        (rank == 4 && (file == 2 || file == 6));
    case 6:
      return ours ? rank <= 4 || ((rank == 5 || rank == 6) && file % 2 == 0)
                  : rank >= 5 || ((rank == 3 || rank == 4) && file % 2 == 0);
    default: return true;
  }
}

struct ThreatMap {
  std::vector<uint32_t> relation;  // [14][90][90] -> first slot, or UINT32_MAX
  uint8_t attacked[90][kPieces];   // slot offset of the attacked piece, 255 = impossible
  uint32_t vocab = 0;
};

// threat_relation_map and threat_attacked_offsets (src/az.rs:577-716): the
// (attacker, source, target) relations a piece could ever have, in attacker,
// source, target order, each followed by one slot per piece that can stand on
// the target.
const ThreatMap& threat_map() {
  static const ThreatMap map = [] {
    ThreatMap m;
    m.relation.assign((size_t)kPieces * kSq * kSq, UINT32_MAX);
    uint32_t next = 0;
    for (int attacker = 0; attacker < kPieces; ++attacker) {
      const bool ours = attacker < 7;
      const int kind = attacker % 7;
      for (int source = 0; source < kSq; ++source) {
        if (!threat_reachable(attacker, source)) continue;
        const int rank = source / 9, file = source % 9;
        int targets[18], n = 0;
        if (kind == 4 || kind == 5) {
          for (int t = 0; t < kSq; ++t)
            if (t != source && (t / 9 == rank || t % 9 == file)) targets[n++] = t;
        } else {
          static const int general[4][2] = {{0, -1}, {0, 1}, {-1, 0}, {1, 0}};
          static const int advisor[4][2] = {{-1, -1}, {1, -1}, {-1, 1}, {1, 1}};
          static const int elephant[4][2] = {{-2, -2}, {2, -2}, {-2, 2}, {2, 2}};
          static const int horse[8][2] = {{-1, -2}, {1, -2}, {-1, 2}, {1, 2}, {-2, -1}, {-2, 1}, {2, -1}, {2, 1}};
          static const int soldier_home_ours[1][2] = {{0, -1}};
          static const int soldier_home_theirs[1][2] = {{0, 1}};
          static const int soldier_across_ours[3][2] = {{0, -1}, {-1, 0}, {1, 0}};
          static const int soldier_across_theirs[3][2] = {{0, 1}, {-1, 0}, {1, 0}};
          const int(*steps)[2] = nullptr;
          int ns = 0;
          switch (kind) {
            case 0: steps = general; ns = 4; break;
            case 1: steps = advisor; ns = 4; break;
            case 2: steps = elephant; ns = 4; break;
            case 3: steps = horse; ns = 8; break;
            default:
              if (ours && rank <= 4) { steps = soldier_across_ours; ns = 3; }
              else if (!ours && rank >= 5) { steps = soldier_across_theirs; ns = 3; }
              else if (ours) { steps = soldier_home_ours; ns = 1; }
              else { steps = soldier_home_theirs; ns = 1; }
          }
          for (int i = 0; i < ns; ++i) {
            const int tf = file + steps[i][0], tr = rank + steps[i][1];
            if (tf < 0 || tf > 8 || tr < 0 || tr > 9) continue;
            if ((kind == 0 || kind == 1) && (tf < 3 || tf > 5 || (ours ? tr < 7 : tr > 2))) continue;
            if (kind == 2 && (ours ? tr < 5 : tr > 4)) continue;
            targets[n++] = tr * 9 + tf;
          }
        }
        for (int i = 0; i < n; ++i) {
          m.relation[((size_t)attacker * kSq + source) * kSq + targets[i]] = next;
          for (int piece = 0; piece < kPieces; ++piece) next += threat_reachable(piece, targets[i]) ? 1 : 0;
        }
      }
    }
    for (int sq = 0; sq < kSq; ++sq) {
      uint8_t k = 0;
      for (int piece = 0; piece < kPieces; ++piece) m.attacked[sq][piece] = threat_reachable(piece, sq) ? k++ : 255;
    }
    m.vocab = next;
    return m;
  }();
  return map;
}

// value_threat_index (src/az.rs:718-742).
uint32_t threat_index(int perspective, int source, int attacker_code, int target, int attacked_code) {
  const ThreatMap& m = threat_map();
  auto piece_index = [&](int code) {
    const int color = code > 0 ? 0 : 1, kind = (code > 0 ? code : -code) - 1;
    return (color == perspective ? 0 : 7) + kind;
  };
  const int a = piece_index(attacker_code), v = piece_index(attacked_code);
  const int cs = canonical_square(perspective, source), ct = canonical_square(perspective, target);
  const uint32_t base = m.relation[((size_t)a * kSq + cs) * kSq + ct];
  if (base == UINT32_MAX) return UINT32_MAX;
  const uint8_t off = m.attacked[ct][v];
  if (off == 255) return UINT32_MAX;
  return base + off;
}

// Position::visit_occupied_attacks (src/xiangqi/mod.rs:286-389): every piece
// attacking an occupied square, sources in square order.
template <class Visit>
void visit_attacks(const int8_t* b, Visit&& visit) {
  auto inside = [](int f, int r) { return f >= 0 && f < 9 && r >= 0 && r < 10; };
  for (int source = 0; source < kSq; ++source) {
    const int v = b[source];
    if (v == 0) continue;
    const int kind = (v > 0 ? v : -v) - 1;
    const bool red = v > 0;
    const int file = source % 9, rank = source / 9;
    auto step = [&](int df, int dr) {
      const int tf = file + df, tr = rank + dr;
      if (inside(tf, tr) && b[tr * 9 + tf] != 0) visit(source, v, tr * 9 + tf, (int)b[tr * 9 + tf]);
    };
    auto in_palace = [&](int f, int r) { return f >= 3 && f <= 5 && (red ? r >= 7 : r <= 2); };
    static const int ortho[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
    switch (kind) {
      case 0:
        for (auto& d : ortho)
          if (inside(file + d[0], rank + d[1]) && in_palace(file + d[0], rank + d[1])) step(d[0], d[1]);
        break;
      case 1: {
        static const int diag[4][2] = {{-1, -1}, {-1, 1}, {1, -1}, {1, 1}};
        for (auto& d : diag)
          if (inside(file + d[0], rank + d[1]) && in_palace(file + d[0], rank + d[1])) step(d[0], d[1]);
        break;
      }
      case 2: {
        static const int el[4][2] = {{-2, -2}, {-2, 2}, {2, -2}, {2, 2}};
        for (auto& d : el) {
          const int tf = file + d[0], tr = rank + d[1];
          if (inside(tf, tr) && (red ? tr >= 5 : tr <= 4) && b[(rank + d[1] / 2) * 9 + file + d[0] / 2] == 0)
            step(d[0], d[1]);
        }
        break;
      }
      case 3: {
        static const int hs[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                                     {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
        for (auto& h : hs)
          if (inside(file + h[2], rank + h[3]) && inside(file + h[0], rank + h[1]) &&
              b[(rank + h[1]) * 9 + file + h[0]] == 0)
            step(h[2], h[3]);
        break;
      }
      case 4:
      case 5:
        for (auto& d : ortho) {
          int tf = file + d[0], tr = rank + d[1], occupied = 0;
          while (inside(tf, tr)) {
            const int t = tr * 9 + tf;
            if (b[t] != 0) {
              ++occupied;
              if (kind == 4 || occupied == 2) {
                visit(source, v, t, (int)b[t]);
                break;
              }
            }
            tf += d[0];
            tr += d[1];
          }
        }
        break;
      default:
        step(0, red ? -1 : 1);
        if (red ? rank <= 4 : rank >= 5) {
          step(-1, 0);
          step(1, 0);
        }
    }
  }
}

// ---- policy move records (src/az.rs:1766-1887) ------------------------------
// Board helpers in absolute coordinates; colour 0 = Red (positive codes).
inline int color_of(int v) { return v > 0 ? 0 : 1; }
inline int kind_of(int v) { return (v > 0 ? v : -v) - 1; }
inline bool on_board(int f, int r) { return f >= 0 && f < 9 && r >= 0 && r < 10; }
inline bool palace(int color, int f, int r) { return f >= 3 && f <= 5 && (color == 0 ? r >= 7 : r <= 2); }

int general_of(const int8_t* b, int color) { return last_general(b, color); }  // last in scan order

// Position::attacked_squares_mask (src/xiangqi/mod.rs:391-484) as a 90-entry
// flag array: squares attacked by `by`, empty or not.
// enemy_general: general_of(b, 1 - by).
void attacked_squares(const int8_t* b, int by, uint8_t* mask, int enemy_general) {
  std::memset(mask, 0, kSq);
  auto mark = [&](int f, int r) {
    if (on_board(f, r)) mask[r * 9 + f] = 1;
  };
  for (int sq = 0; sq < kSq; ++sq) {
    const int v = b[sq];
    if (v == 0 || color_of(v) != by) continue;
    const int f = sq % 9, r = sq / 9;
    switch (kind_of(v)) {
      case 0: {
        static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
        for (auto& d : o)
          if (on_board(f + d[0], r + d[1]) && palace(by, f + d[0], r + d[1])) mark(f + d[0], r + d[1]);
        if (enemy_general >= 0 && enemy_general % 9 == f) {
          bool clear = true;
          const int lo = std::min(r, enemy_general / 9), hi = std::max(r, enemy_general / 9);
          for (int rr = lo + 1; rr < hi; ++rr) clear &= b[rr * 9 + f] == 0;
          if (clear) mask[enemy_general] = 1;
        }
        break;
      }
      case 1: {
        static const int d4[4][2] = {{-1, -1}, {-1, 1}, {1, -1}, {1, 1}};
        for (auto& d : d4)
          if (on_board(f + d[0], r + d[1]) && palace(by, f + d[0], r + d[1])) mark(f + d[0], r + d[1]);
        break;
      }
      case 2: {
        static const int e[4][2] = {{-2, -2}, {-2, 2}, {2, -2}, {2, 2}};
        for (auto& d : e) {
          const int tf = f + d[0], tr = r + d[1];
          if (on_board(tf, tr) && (by == 0 ? tr >= 5 : tr <= 4) && b[(r + d[1] / 2) * 9 + f + d[0] / 2] == 0)
            mark(tf, tr);
        }
        break;
      }
      case 3: {
        static const int hs[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                                     {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
        for (auto& h : hs)
          if (on_board(f + h[2], r + h[3]) && b[(r + h[1]) * 9 + f + h[0]] == 0) mark(f + h[2], r + h[3]);
        break;
      }
      case 4:
      case 5: {
        static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
        const bool rook = kind_of(v) == 4;
        for (auto& d : o) {
          int tf = f + d[0], tr = r + d[1], blockers = 0;
          while (on_board(tf, tr)) {
            const bool occupied = b[tr * 9 + tf] != 0;
            if (rook) {
              mark(tf, tr);
              if (occupied) break;
            } else {
              if (blockers == 1) mark(tf, tr);  // beyond the screen, up to the next piece
              if (occupied && ++blockers == 2) break;
            }
            tf += d[0];
            tr += d[1];
          }
        }
        break;
      }
      default:
        mark(f, r + (by == 0 ? -1 : 1));
        if (by == 0 ? r <= 4 : r >= 5) {
          mark(f - 1, r);
          mark(f + 1, r);
        }
    }
  }
}

// Position::gives_check_after_move_fast (src/xiangqi/mod.rs:763-1012).
// g: the square of the general of 1 - side (general_of), -1 if none.
bool gives_check(const int8_t* b, int side, int from, int to, int g) {
  if (g < 0 || b[from] == 0) return false;
  const int moving = b[from];
  auto occ = [&](int sq) -> int { return sq == from ? 0 : (sq == to ? moving : (int)b[sq]); };
  auto between = [&](int a, int c) -> int {  // pieces strictly between, INT_MAX-like if not aligned
    if (a % 9 == c % 9) {
      int n = 0;
      for (int r = std::min(a / 9, c / 9) + 1; r < std::max(a / 9, c / 9); ++r) n += occ(r * 9 + a % 9) != 0;
      return n;
    }
    if (a / 9 == c / 9) {
      int n = 0;
      for (int f = std::min(a % 9, c % 9) + 1; f < std::max(a % 9, c % 9); ++f) n += occ((a / 9) * 9 + f) != 0;
      return n;
    }
    return 1 << 20;
  };
  // piece_attacks_virtual (src/xiangqi/mod.rs:920-979) of the moved piece.
  {
    const int pf = to % 9, pr = to / 9, tf = g % 9, tr = g / 9, df = tf - pf, dr = tr - pr;
    const int color = color_of(moving);
    bool hit = false;
    switch (kind_of(moving)) {
      case 0:
        hit = (std::abs(df) + std::abs(dr) == 1 && palace(color, tf, tr)) ||
              (pf == tf && occ(g) != 0 && kind_of(occ(g)) == 0 && color_of(occ(g)) != color && between(to, g) == 0);
        break;
      case 1: hit = std::abs(df) == 1 && std::abs(dr) == 1 && palace(color, tf, tr); break;
      case 2:
        hit = std::abs(df) == 2 && std::abs(dr) == 2 && (color == 0 ? tr >= 5 : tr <= 4) &&
              occ(((pr + tr) / 2) * 9 + (pf + tf) / 2) == 0;
        break;
      case 3: {
        static const int hs[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                                     {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
        for (auto& h : hs)
          if (df == h[2] && dr == h[3]) {
            hit = occ((pr + h[1]) * 9 + pf + h[0]) == 0;
            break;
          }
        break;
      }
      case 4: hit = (pf == tf || pr == tr) && between(to, g) == 0; break;
      case 5: hit = (pf == tf || pr == tr) && between(to, g) == 1; break;
      default:
        hit = (tf == pf && tr == pr + (color == 0 ? -1 : 1)) ||
              ((color == 0 ? tr <= 4 : tr >= 5) && tr == pr && std::abs(df) == 1);
    }
    if (hit) return true;
  }
  // discovered checks along the orthogonal rays through from or to.
  static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
  const int gf = g % 9, gr = g / 9;
  auto on_ray = [&](int q, int df, int dr) {
    const int qf = q % 9, qr = q / 9;
    return dr == 0 ? (qr == gr && (qf - gf) * df > 0) : (qf == gf && (qr - gr) * dr > 0);
  };
  for (auto& d : o) {
    if (!on_ray(from, d[0], d[1]) && !on_ray(to, d[0], d[1])) continue;
    int nf = gf + d[0], nr = gr + d[1];
    bool screen = false;
    while (on_board(nf, nr)) {
      const int p = occ(nr * 9 + nf);
      if (p != 0) {
        if (!screen) {
          if (color_of(p) == side && (kind_of(p) == 4 || (kind_of(p) == 0 && d[0] == 0))) return true;
          screen = true;
        } else if (color_of(p) == side && kind_of(p) == 5) {
          return true;
        } else {
          break;
        }
      }
      nf += d[0];
      nr += d[1];
    }
  }
  // a horse or elephant whose leg / eye was `from` (leaper_revealed_*, :845-918).
  // Every leg or eye of a leap onto the general is one of its four diagonal
  // neighbours, so no other `from` can reveal one.
  if (std::abs(from % 9 - gf) != 1 || std::abs(from / 9 - gr) != 1) return false;
  static const int hs[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                               {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
  for (auto& h : hs) {
    const int of = gf - h[2], orr = gr - h[3];
    if (!on_board(of, orr) || !on_board(of + h[0], orr + h[1])) continue;
    const int p = occ(orr * 9 + of);
    if ((orr + h[1]) * 9 + of + h[0] == from && p != 0 && kind_of(p) == 3 && color_of(p) == side) return true;
  }
  static const int es[4][4] = {{1, 1, 2, 2}, {1, -1, 2, -2}, {-1, 1, -2, 2}, {-1, -1, -2, -2}};
  for (auto& e : es) {
    const int of = gf - e[2], orr = gr - e[3];
    if (!on_board(of, orr) || !on_board(of + e[0], orr + e[1])) continue;
    const int p = occ(orr * 9 + of);
    if ((orr + e[1]) * 9 + of + e[0] == from && p != 0 && kind_of(p) == 2 && color_of(p) == side &&
        (side == 0 ? gr >= 5 : gr <= 4))
      return true;
  }
  return false;
}

// ---- training batch packer (PackedBatch::from_indices, src/az/dataloader.rs:113-336)
constexpr int64_t kSparseTable = 2396815;    // POLICY_SPARSE_TABLE_SIZE (src/az.rs:77-78)
constexpr int64_t kSparseMain = 2086 * 14 * 81;
constexpr int64_t kTacticalExact = 2086 * 7 * 64;  // POLICY_TACTICAL_EXACT_SIZE (src/az.rs:66-67)
constexpr int64_t kTacticalSize = kTacticalExact + 7 * 64;
constexpr float kPolicyMask = -1.0e9f;       // POLICY_MASK_VALUE (src/az/dataloader.rs:22)
constexpr uint32_t kPad = 0xffffffffu;

struct RowDims {
  int features = 0, moves = 0, threats = 0;
};

// The canonical position of a sample (Position::from_canonical_piece_squares,
// src/xiangqi/mod.rs:112-157): own pieces (index < 7) Red, others Black, Red
// to move; board_features[sq] = the feature standing on sq (-1 if none).
void sample_board(const uint16_t* f, int n, int8_t* board, int* board_features) {
  std::memset(board, 0, kSq);
  for (int sq = 0; sq < kSq; ++sq) board_features[sq] = -1;
  for (int k = 0; k < n; ++k) {
    if (f[k] >= CNNUE_AZ_INPUT) continue;
    const int pi = f[k] / kSq, sq = f[k] % kSq;
    board[sq] = (int8_t)(pi < 7 ? pi + 1 : -(pi - 7 + 1));
    board_features[sq] = f[k];
  }
}

// canonical_general_buckets_from_features (src/az.rs:168-184): the last
// general of each side in feature order.
void sample_buckets(const uint16_t* f, int n, int* us, int* them) {
  *us = 4;
  *them = 4;
  for (int k = 0; k < n; ++k) {
    if (f[k] >= CNNUE_AZ_INPUT) continue;
    const int pi = f[k] / kSq, sq = f[k] % kSq;
    if (pi == 0) *us = general_bucket(0, sq);
    if (pi == 7) *them = general_bucket(7, sq);
  }
}

// value_threat_features (src/az/dataloader.rs:307-326).
int sample_threats(const int8_t* board, uint32_t* out) {
  int n = 0;
  visit_attacks(board, [&](int source, int attacker, int target, int attacked) {
    const uint32_t f = threat_index(0, source, attacker, target, attacked);
    if (f != UINT32_MAX && n < CNNUE_AZ_THREAT_MAX) out[n++] = f;
  });
  return n;
}

// policy_king_distance_buckets (src/az.rs:841-859).
void king_distance(int from, int to, int them, int* distance, int* approach) {
  const int king = kSq - 1 - ((7 + them / 3) * 9 + 3 + them % 3);
  const int before = std::abs(from / 9 - king / 9) + std::abs(from % 9 - king % 9);
  const int after = std::abs(to / 9 - king / 9) + std::abs(to % 9 - king % 9);
  *approach = std::min(std::max(before - after, -2), 2) + 2;
  *distance = std::min(after, 5);
}

void pack_row(const cnnue_az_samples* s, int64_t sample, int64_t row, const RowDims& dims,
              const uint32_t* threats, int n_threats, const cnnue_az_packed* o) {
  const uint16_t* f = s->features + s->feature_offsets[sample];
  const int nf = (int)(s->feature_offsets[sample + 1] - s->feature_offsets[sample]);
  const int F = dims.features, M = dims.moves, T = dims.threats;
  int us, them;
  sample_buckets(f, nf, &us, &them);
  // pack_features (:193-205): padding where a feature is out of range
  uint32_t* fi = o->feature_items + row * F;
  for (int k = 0; k < F; ++k) fi[k] = k < nf && f[k] < CNNUE_AZ_INPUT ? pack(f[k], us, them) : kPad;
  uint32_t* ti = o->value_threat_indices + row * T;
  for (int k = 0; k < T; ++k) ti[k] = k < n_threats ? threats[k] : kPad;
  // pack_policy (:207-305)
  int8_t board[kSq];
  int bf[kSq];
  sample_board(f, nf, board, bf);
  uint8_t opp[kSq], own[kSq];
  const int enemy_general = general_of(board, 1);
  attacked_squares(board, 1, opp, general_of(board, 0));
  attacked_squares(board, 0, own, enemy_general);
  const auto& moves = dense_moves();
  const bool compact = o->policy_sparse_indices == nullptr;
  int64_t* items = o->policy_items + row * M;
  float* targets = o->policy_targets + row * M;
  int64_t* sparse = compact ? nullptr : o->policy_sparse_indices + row * M * 7;
  int64_t* tactical = compact ? nullptr : o->policy_tactical_indices + row * M * 2;
  float* mask = compact ? nullptr : o->policy_mask + row * M;
  uint8_t* signature = compact ? o->policy_signature + row * M : nullptr;
  if (compact) o->king_buckets[row] = (uint8_t)(us | them << 4);
  for (int k = 0; k < M; ++k) {
    items[k] = 0;
    targets[k] = 0.f;
    if (compact) {
      signature[k] = 0;
      continue;
    }
    mask[k] = kPolicyMask;
    for (int j = 0; j < 7; ++j) sparse[k * 7 + j] = kSparseTable - 1;
    tactical[k * 2] = tactical[k * 2 + 1] = kTacticalSize;
  }
  const uint32_t m0 = s->move_offsets[sample], m1 = s->move_offsets[sample + 1];
  int off = 0;
  for (uint32_t j = m0; j < m1; ++j) {
    const int mi = s->move_indices[j];
    if (mi >= kDenseMoves) continue;
    const float target = s->policy[j];
    targets[off] = std::fmax(target, 0.f);
    if (!compact) mask[off] = 0.f;
    const int from = moves[mi] / kSq, to = moves[mi] % kSq;
    const int mf = bf[from];
    const bool move_valid = mf >= 0 && mf / kSq < 7;
    int64_t cf = 0, ct = 0, cc = 0;
    bool capture = false;
    if (move_valid) {
      cf = mf;
      ct = (int64_t)(mf / kSq) * kSq + to;
      if (bf[to] >= 0) {
        cc = bf[to];
        capture = true;
      }
    }
    // pack_policy_item (src/az/fused_policy.rs:146-157)
    items[off] = (int64_t)((uint64_t)mi | (uint64_t)cf << 12 | (uint64_t)ct << 23 | (uint64_t)cc << 34 |
                           (uint64_t)move_valid << 45 | (uint64_t)capture << 46 | (uint64_t)1 << 47);
    if (move_valid && compact) {
      signature[off] = (uint8_t)(opp[from] | opp[to] << 1 | own[from] << 2 | own[to] << 3 | (int)capture << 4 |
                                 (int)gives_check(board, 0, from, to, enemy_general) << 5);
    } else if (move_valid) {
      const int piece = mf / kSq;
      const int pair = us * 9 + them;
      int64_t* sp = sparse + off * 7;
      // policy_sparse_main_index / _capture_index / _factor_indices (src/az.rs:763-813)
      sp[0] = (((int64_t)mi * 14 + piece) * 9 + us) * 9 + them;
      sp[1] = kSparseMain + (int64_t)mi * 15 + (capture ? cc / kSq : 14);
      int distance, approach;
      king_distance(from, to, them, &distance, &approach);
      const int64_t move_piece = (int64_t)kDenseMoves * 14, move_king = (int64_t)kDenseMoves * 81;
      const int64_t distance_off = move_piece + move_king + 14 * 81;
      sp[2] = kSparseTable + (int64_t)mi * 14 + piece;
      sp[3] = kSparseTable + move_piece + (int64_t)mi * 81 + pair;
      sp[4] = kSparseTable + move_piece + move_king + piece * 81 + pair;
      sp[5] = kSparseTable + distance_off + piece * 6 + distance;
      sp[6] = kSparseTable + distance_off + 14 * 6 + piece * 5 + approach;
      // policy_tactical_indices (src/az.rs:815-839)
      const int64_t sig = (int64_t)opp[from] | (int64_t)opp[to] << 1 | (int64_t)own[from] << 2 |
                          (int64_t)own[to] << 3 | (int64_t)capture << 4 |
                          (int64_t)gives_check(board, 0, from, to, enemy_general) << 5;
      tactical[off * 2] = ((int64_t)mi * 7 + piece) * 64 + sig;
      tactical[off * 2 + 1] = kTacticalExact + piece * 64 + sig;
    }
    ++off;
  }
  // normalize_policy_targets (:432-446)
  if (off > 0) {
    float sum = 0.f;
    for (int k = 0; k < off; ++k) sum += targets[k];
    if (std::isfinite(sum) && sum > 1.0e-12f) {
      for (int k = 0; k < off; ++k) targets[k] = std::fmax(targets[k] / sum, 0.f);
    } else {
      const float uniform = 1.0f / (float)off;
      for (int k = 0; k < off; ++k) targets[k] = uniform;
    }
  }
  // normalize_wdl_target (src/az.rs:2586-2599)
  float w[3];
  for (int k = 0; k < 3; ++k) w[k] = std::fmax(s->value_wdl[sample * 3 + k], 0.f);
  const float wsum = w[0] + w[1] + w[2];
  if (std::isfinite(wsum) && wsum > 1.0e-6f) {
    for (int k = 0; k < 3; ++k) o->value_wdl[row * 3 + k] = w[k] / wsum;
  } else {
    o->value_wdl[row * 3] = 0.f;
    o->value_wdl[row * 3 + 1] = 1.f;
    o->value_wdl[row * 3 + 2] = 0.f;
  }
  o->values[row] = std::min(std::max(s->value[sample], -1.0f), 1.0f);
  for (int k = 0; k < CNNUE_AZ_RULE_CONTEXT; ++k)
    o->rule_context[row * CNNUE_AZ_RULE_CONTEXT + k] = s->rule_context[sample * CNNUE_AZ_RULE_CONTEXT + k];
  o->policy_weights[row] = std::fmax(s->policy_weight[sample], 0.f);
  o->value_weights[row] = std::fmax(s->value_weight[sample], 0.f);
  const uint32_t ply = s->ply[sample];
  const int phase = ply < 40 ? 0 : (ply < 120 ? 1 : 2);
  for (int k = 0; k < 3; ++k) o->value_phase_masks[row * 3 + k] = k == phase ? 1.f : 0.f;
}

template <class Fn>
void parallel_rows(int64_t n, int n_threads, Fn&& fn) {
  int t = n_threads > 0 ? n_threads : (int)std::min<unsigned>(std::max(1u, std::thread::hardware_concurrency()), 16u);
  t = (int)std::min<int64_t>(t, std::max<int64_t>(n / 16, 1));
  if (t <= 1) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(t);
  for (int k = 0; k < t; ++k)
    pool.emplace_back([&, k] {
      for (int64_t i = n * k / t; i < n * (k + 1) / t; ++i) fn(i);
    });
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

int cnnue_az_policy_moves(const int8_t* board, int side, const uint8_t* moves, int n_moves, uint32_t* info) {
  if (!moves || !info || n_moves < 0) return set_error(CNNUE_ERR_INVALID_ARG, "null moves or info");
  if (side != 0 && side != 1) return set_error(CNNUE_ERR_INVALID_ARG, "side %d", side);
  if (int st = check_board(board)) return st;
  static const std::vector<uint16_t> s2d = [] {
    std::vector<uint16_t> v(kSq * kSq, 0xffff);
    const auto& d = dense_moves();
    for (size_t i = 0; i < d.size(); ++i) v[d[i]] = (uint16_t)i;
    return v;
  }();
  uint8_t opp[kSq], own[kSq];
  const int enemy_general = general_of(board, 1 - side);
  attacked_squares(board, 1 - side, opp, general_of(board, side));
  attacked_squares(board, side, own, enemy_general);
  int us, them;
  buckets_of(board, side, &us, &them);
  int status = CNNUE_OK;
  for (int i = 0; i < n_moves; ++i) {
    const int from = moves[2 * i], to = moves[2 * i + 1];
    if (from >= kSq || to >= kSq || board[from] == 0) {
      status = set_error(CNNUE_ERR_INVALID_ARG, "move %d: %d -> %d has no piece to move", i, from, to);
      info[2 * i] = info[2 * i + 1] = 0xffffffffu;
      continue;
    }
    const int cf = canonical_square(side, from), ct = canonical_square(side, to);
    const uint32_t dense = s2d[cf * kSq + ct];
    const int moved = (color_of(board[from]) == side ? 0 : 7) + kind_of(board[from]);
    const int captured = board[to] != 0 ? (color_of(board[to]) == side ? 0 : 7) + kind_of(board[to]) : 15;
    const uint32_t sig = (uint32_t)opp[from] | (uint32_t)opp[to] << 1 | (uint32_t)own[from] << 2 |
                         (uint32_t)own[to] << 3 | (uint32_t)(board[to] != 0) << 4 |
                         (uint32_t)gives_check(board, side, from, to, enemy_general) << 5;
    info[2 * i] = (dense == 0xffff ? 0xfffu : dense) | (uint32_t)moved << 12 | (uint32_t)captured << 16 | sig << 20;
    info[2 * i + 1] = (uint32_t)cf | (uint32_t)ct << 7 | (uint32_t)us << 14 | (uint32_t)them << 18;
  }
  return status;
}

int cnnue_az_threat_vocab(void) { return (int)threat_map().vocab; }

int cnnue_az_threat_features(const int8_t* board, int perspective, uint32_t* features, int* count) {
  if (!features || !count) return set_error(CNNUE_ERR_INVALID_ARG, "null features or count");
  if (perspective != 0 && perspective != 1) return set_error(CNNUE_ERR_INVALID_ARG, "perspective %d", perspective);
  if (int st = check_board(board)) return st;
  int n = 0;
  visit_attacks(board, [&](int source, int attacker, int target, int attacked) {
    const uint32_t f = threat_index(perspective, source, attacker, target, attacked);
    if (f != UINT32_MAX && n < CNNUE_AZ_THREAT_MAX) features[n++] = f;
  });
  *count = n;
  return CNNUE_OK;
}

int cnnue_az_quantize(cnnue_az_weights* w) {
  if (!w) return set_error(CNNUE_ERR_INVALID_ARG, "null weights");
  try {
    return quantize(*w);
  } catch (const std::bad_alloc&) {
    return set_error(CNNUE_ERR_INVALID_ARG, "out of host memory");
  }
}

int cnnue_az_quant_table(const cnnue_az_weights* w, int which, const void** data, int64_t* count, float* scale) {
  if (!w || !data) return set_error(CNNUE_ERR_INVALID_ARG, "null weights or data");
  if (which < 0 || which > CNNUE_AZ_Q_CAPTURE) return set_error(CNNUE_ERR_INVALID_ARG, "quantised table %d", which);
  if (which < 4) {
    *data = w->q8[which].data();
    if (count) *count = (int64_t)w->q8[which].size();
    if (scale) *scale = w->scale[which];
  } else {
    *data = w->q32[which - 4].data();
    if (count) *count = (int64_t)w->q32[which - 4].size();
    if (scale) *scale = 1.f;
  }
  return CNNUE_OK;
}

int cnnue_az_quant_flags(const cnnue_az_weights* w, int* value_threat_active, int* policy_tactical_active) {
  if (!w) return set_error(CNNUE_ERR_INVALID_ARG, "null weights");
  if (value_threat_active) *value_threat_active = w->value_threat_active;
  if (policy_tactical_active) *policy_tactical_active = w->policy_tactical_active;
  return CNNUE_OK;
}

int cnnue_az_dense_moves(uint16_t* dense_to_sparse, uint16_t* sparse_to_dense) {
  const auto& moves = dense_moves();
  if (dense_to_sparse) std::copy(moves.begin(), moves.end(), dense_to_sparse);
  if (sparse_to_dense) {
    std::fill(sparse_to_dense, sparse_to_dense + kSq * kSq, (uint16_t)0xffff);
    for (size_t i = 0; i < moves.size(); ++i) sparse_to_dense[moves[i]] = (uint16_t)i;
  }
  return CNNUE_OK;
}


int cnnue_az_board_from_fen(const char* fen, int8_t* board, int* side) {
  if (!fen || !board || !side) return set_error(CNNUE_ERR_INVALID_ARG, "null fen, board or side");
  int8_t b[kSq] = {0};
  const char* p = fen;
  while (*p == ' ' || *p == '\t') ++p;
  int rank = 0, file = 0;
  for (; *p && *p != ' ' && *p != '\t'; ++p) {
    const char c = *p;
    if (c == '/') {
      if (file != 9) return set_error(CNNUE_ERR_FORMAT, "rank %d does not contain 9 files", rank);
      if (++rank >= 10) return set_error(CNNUE_ERR_FORMAT, "expected 10 ranks in FEN");
      file = 0;
      continue;
    }
    if (c >= '0' && c <= '9') {
      file += c - '0';
      continue;
    }
    const char l = (c >= 'A' && c <= 'Z') ? (char)(c - 'A' + 'a') : c;
    int kind;
    switch (l) {
      case 'k': kind = 0; break;
      case 'a': kind = 1; break;
      case 'b': case 'e': kind = 2; break;
      case 'n': case 'h': kind = 3; break;
      case 'r': kind = 4; break;
      case 'c': kind = 5; break;
      case 'p': kind = 6; break;
      default: return set_error(CNNUE_ERR_FORMAT, "invalid piece: %c", c);
    }
    if (file >= 9) return set_error(CNNUE_ERR_FORMAT, "file overflow in FEN");
    b[rank * 9 + file] = (int8_t)((c >= 'A' && c <= 'Z') ? kind + 1 : -(kind + 1));
    ++file;
  }
  if (rank != 9) return set_error(CNNUE_ERR_FORMAT, "expected 10 ranks in FEN");
  if (file != 9) return set_error(CNNUE_ERR_FORMAT, "rank %d does not contain 9 files", rank);
  while (*p == ' ' || *p == '\t') ++p;
  int s = 0;
  if (*p) {
    const char* q = p;
    while (*q && *q != ' ' && *q != '\t') ++q;
    const std::string tok(p, q);
    if (tok == "w" || tok == "r") s = 0;
    else if (tok == "b") s = 1;
    else return set_error(CNNUE_ERR_FORMAT, "invalid side to move: %s", tok.c_str());
  }
  memcpy(board, b, sizeof(b));
  *side = s;
  return CNNUE_OK;
}

int cnnue_az_features(const int8_t* board, int perspective, uint32_t* items, int* count) {
  if (!items || !count) return set_error(CNNUE_ERR_INVALID_ARG, "null items or count");
  if (perspective != 0 && perspective != 1) return set_error(CNNUE_ERR_INVALID_ARG, "perspective %d", perspective);
  int st = check_board(board);
  if (st) return st;
  *count = features(board, perspective, items);
  return CNNUE_OK;
}

int cnnue_az_move_items(const int8_t* board, int from, int to, int perspective, uint32_t* delta,
                        uint8_t* refresh, uint32_t* items, int* count) {
  if (!delta || !refresh || !items || !count)
    return set_error(CNNUE_ERR_INVALID_ARG, "null delta, refresh, items or count");
  if (perspective != 0 && perspective != 1) return set_error(CNNUE_ERR_INVALID_ARG, "perspective %d", perspective);
  int st = check_board(board);
  if (st) return st;
  if (from < 0 || from >= kSq || to < 0 || to >= kSq || from == to)
    return set_error(CNNUE_ERR_INVALID_ARG, "move %d -> %d", from, to);
  if (board[from] == 0) return set_error(CNNUE_ERR_INVALID_ARG, "no piece on square %d", from);
  int8_t after[kSq];
  memcpy(after, board, sizeof(after));
  after[to] = after[from];
  after[from] = 0;
  int us0, them0, us1, them1;
  buckets_of(board, perspective, &us0, &them0);
  buckets_of(after, perspective, &us1, &them1);
  delta[0] = delta[1] = delta[2] = CNNUE_AZ_NO_ITEM;
  if (us0 != us1 || them0 != them1) {
    *refresh = 1;
    *count = features(after, perspective, items);
    return CNNUE_OK;
  }
  *refresh = 0;
  *count = 0;
  delta[0] = pack(feature_of(board[from], from, perspective), us0, them0);
  if (board[to] != 0) delta[1] = pack(feature_of(board[to], to, perspective), us0, them0);
  delta[2] = pack(feature_of(board[from], to, perspective), us1, them1);
  return CNNUE_OK;
}

int cnnue_az_tensor_info(int index, int64_t hidden, const char** name, int64_t* count) {
  if (index < 0 || index >= CNNUE_AZ_TENSORS) return set_error(CNNUE_ERR_INVALID_ARG, "tensor index %d", index);
  if (hidden <= 0) return set_error(CNNUE_ERR_INVALID_ARG, "hidden %lld", (long long)hidden);
  if (name) *name = kSpecs[index].name;
  if (count) *count = count_of(index, hidden);
  return CNNUE_OK;
}

int cnnue_az_weights_random(int64_t hidden, uint64_t seed, cnnue_az_weights** out) {
  if (!out) return set_error(CNNUE_ERR_INVALID_ARG, "null out");
  *out = nullptr;
  if (hidden <= 0 || hidden > (1 << 20)) return set_error(CNNUE_ERR_INVALID_ARG, "invalid hidden_size %lld", (long long)hidden);
  std::unique_ptr<cnnue_az_weights> w(new (std::nothrow) cnnue_az_weights);
  if (!w) return set_error(CNNUE_ERR_INVALID_ARG, "out of host memory");
  w->hidden = hidden;
  try {
    for (int i = 0; i < CNNUE_AZ_TENSORS; ++i) w->t[i].assign((size_t)count_of(i, hidden), 0.0f);
  } catch (const std::bad_alloc&) {
    return set_error(CNNUE_ERR_INVALID_ARG, "out of host memory");
  }
  // Draw order of random_with_arch: input_hidden, value_head_hidden,
  // value_threat_embedding, policy_context_hidden, policy_accumulator_hidden;
  // every other tensor starts at zero.
  SplitMix rng{seed};
  const float head_scale = std::sqrt(2.0f / (float)hidden) * 0.5f;
  for (float& x : w->t[0]) x = rng.weight(0.015f);
  for (float& x : w->t[7]) x = rng.weight(head_scale);
  for (float& x : w->t[10]) x = rng.weight(0.02f);
  for (float& x : w->t[15]) x = rng.weight(head_scale);
  for (float& x : w->t[17]) x = rng.weight(head_scale);
  if (int st = cnnue_az_quantize(w.get())) return st;
  *out = w.release();
  return CNNUE_OK;
}

int cnnue_az_weights_load(const char* path, cnnue_az_weights** out) {
  if (!path || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null path or out");
  *out = nullptr;
  std::vector<char> bytes;
  int st = read_file(path, bytes);
  if (st) return st;
  std::map<std::string, TensorRef> tensors;
  const char* data = nullptr;
  if ((st = parse_safetensors(bytes, tensors, &data))) return st;
  std::vector<float> version;
  if ((st = load_f32(tensors, data, "az_model_format_version", version))) return st;
  if (version.empty()) return set_error(CNNUE_ERR_FORMAT, "missing AZ model format");
  if (version[0] != CNNUE_AZ_FORMAT_VERSION)
    return set_error(CNNUE_ERR_FORMAT, "unsupported AZ model format %g; expected v%g", (double)version[0],
                     (double)CNNUE_AZ_FORMAT_VERSION);
  std::unique_ptr<cnnue_az_weights> w(new (std::nothrow) cnnue_az_weights);
  if (!w) return set_error(CNNUE_ERR_IO, "out of host memory");
  if ((st = load_f32(tensors, data, "hidden_bias", w->t[6]))) return st;
  w->hidden = (int64_t)w->t[6].size();
  if (w->hidden == 0) return set_error(CNNUE_ERR_FORMAT, "aznnue arch invalid: invalid hidden_size 0");
  for (int i = 0; i < CNNUE_AZ_TENSORS; ++i) {
    if (i != 6 && (st = load_f32(tensors, data, kSpecs[i].name, w->t[i]))) return st;
    const int64_t expected = count_of(i, w->hidden);
    if ((int64_t)w->t[i].size() != expected)
      return set_error(CNNUE_ERR_FORMAT, "az model tensor `%s` length mismatch: got %lld, expected %lld",
                       kSpecs[i].name, (long long)w->t[i].size(), (long long)expected);
  }
  if ((st = cnnue_az_quantize(w.get()))) return st;
  *out = w.release();
  return CNNUE_OK;
}

int cnnue_az_weights_save(const cnnue_az_weights* w, const char* path) {
  if (!w || !path) return set_error(CNNUE_ERR_INVALID_ARG, "null weights or path");
  struct Entry {
    std::vector<int64_t> shape;
    const float* data;
    uint64_t n;
  };
  static const float kVersion = CNNUE_AZ_FORMAT_VERSION;
  std::map<std::string, Entry> entries;
  entries["az_model_format_version"] = Entry{{1}, &kVersion, 1};
  for (int i = 0; i < CNNUE_AZ_TENSORS; ++i)
    entries[kSpecs[i].name] = Entry{shape_of(i, w->hidden), w->t[i].data(), (uint64_t)w->t[i].size()};
  std::string header = "{";
  uint64_t offset = 0;
  bool first = true;
  for (const auto& e : entries) {
    if (!first) header += ",";
    first = false;
    header += "\"" + e.first + "\":{\"dtype\":\"F32\",\"shape\":[";
    for (size_t d = 0; d < e.second.shape.size(); ++d) {
      if (d) header += ",";
      header += std::to_string(e.second.shape[d]);
    }
    header += "],\"data_offsets\":[" + std::to_string(offset) + "," + std::to_string(offset + 4 * e.second.n) + "]}";
    offset += 4 * e.second.n;
  }
  header += "}";
  while (header.size() % 8) header += ' ';
  File f(fopen(path, "wb"));
  if (!f) return set_error(CNNUE_ERR_IO, "cannot open %s for writing", path);
  uint8_t len[8];
  for (int i = 0; i < 8; ++i) len[i] = (uint8_t)((uint64_t)header.size() >> (8 * i));
  bool ok = fwrite(len, 1, 8, f.get()) == 8 && fwrite(header.data(), 1, header.size(), f.get()) == header.size();
  for (const auto& e : entries)
    ok = ok && (e.second.n == 0 || fwrite(e.second.data, 4, e.second.n, f.get()) == e.second.n);
  FILE* raw = f.release();
  ok = (fclose(raw) == 0) && ok;
  if (!ok) return set_error(CNNUE_ERR_IO, "short write on %s", path);
  return CNNUE_OK;
}

int cnnue_az_weights_destroy(cnnue_az_weights* w) {
  delete w;
  return CNNUE_OK;
}

int64_t cnnue_az_weights_hidden(const cnnue_az_weights* w) { return w ? w->hidden : 0; }

int cnnue_az_weights_tensor(cnnue_az_weights* w, int index, float** data, int64_t* count) {
  if (!w || !data) return set_error(CNNUE_ERR_INVALID_ARG, "null weights or data");
  if (index < 0 || index >= CNNUE_AZ_TENSORS) return set_error(CNNUE_ERR_INVALID_ARG, "tensor index %d", index);
  *data = w->t[index].data();
  if (count) *count = (int64_t)w->t[index].size();
  return CNNUE_OK;
}

int cnnue_az_pack_batch(const cnnue_az_samples* s, const int64_t* rows, int64_t batch, int64_t cap_features,
                        int64_t cap_moves, int64_t cap_threats, int fixed_strides, cnnue_az_packed* out,
                        int n_threads) {
  if (!s || !out || batch < 0) return set_error(CNNUE_ERR_INVALID_ARG, "null samples/out or negative batch");
  if (s->n < 0 || (s->n > 0 && (!s->feature_offsets || !s->move_offsets)))
    return set_error(CNNUE_ERR_INVALID_ARG, "samples without offsets");
  for (int64_t r = 0; r < batch; ++r) {
    const int64_t i = rows ? rows[r] : r;
    if (i < 0 || i >= s->n) return set_error(CNNUE_ERR_INVALID_ARG, "batch row %lld: sample %lld of %lld",
                                             (long long)r, (long long)i, (long long)s->n);
  }
  // pass 1: per-row counts and threat features (the batch maxima set the strides)
  std::vector<RowDims> dims(batch);
  std::vector<uint32_t> threats((size_t)batch * CNNUE_AZ_THREAT_MAX);
  parallel_rows(batch, n_threads, [&](int64_t r) {
    const int64_t i = rows ? rows[r] : r;
    const uint16_t* f = s->features + s->feature_offsets[i];
    const int nf = (int)(s->feature_offsets[i + 1] - s->feature_offsets[i]);
    int8_t board[kSq];
    int bf[kSq];
    sample_board(f, nf, board, bf);
    dims[r].features = nf;
    dims[r].threats = sample_threats(board, threats.data() + (size_t)r * CNNUE_AZ_THREAT_MAX);
    int m = 0;
    for (uint32_t j = s->move_offsets[i]; j < s->move_offsets[i + 1]; ++j) m += s->move_indices[j] < kDenseMoves;
    dims[r].moves = m;
  });
  RowDims mx;
  mx.features = mx.moves = mx.threats = 1;  // .max(1) (:116-136)
  for (const RowDims& d : dims) {
    mx.features = std::max(mx.features, d.features);
    mx.moves = std::max(mx.moves, d.moves);
    mx.threats = std::max(mx.threats, d.threats);
  }
  out->batch = batch;
  out->max_features = mx.features;
  out->max_policy_moves = mx.moves;
  out->max_value_threats = mx.threats;
  if (mx.features > cap_features || mx.moves > cap_moves || mx.threats > cap_threats)
    return set_error(CNNUE_ERR_WORKSPACE, "batch needs %d features, %d moves, %d threats per row", mx.features,
                     mx.moves, mx.threats);
  if (fixed_strides) {  // the capacities are the strides (static shapes for a captured step)
    mx.features = (int)cap_features;
    mx.moves = (int)cap_moves;
    mx.threats = (int)cap_threats;
    out->max_features = cap_features;
    out->max_policy_moves = cap_moves;
    out->max_value_threats = cap_threats;
  }
  if (batch == 0) return CNNUE_OK;
  const bool compact = !out->policy_sparse_indices && !out->policy_tactical_indices && !out->policy_mask;
  if (!out->feature_items || !out->value_threat_indices || !out->policy_items || !out->policy_targets ||
      !out->value_wdl || !out->values || !out->rule_context || !out->policy_weights || !out->value_weights ||
      !out->value_phase_masks)
    return set_error(CNNUE_ERR_INVALID_ARG, "null output array");
  if (compact ? (!out->policy_signature || !out->king_buckets)
              : (!out->policy_sparse_indices || !out->policy_tactical_indices || !out->policy_mask))
    return set_error(CNNUE_ERR_INVALID_ARG, "give all of sparse/tactical/mask, or the compact signature + buckets");
  parallel_rows(batch, n_threads, [&](int64_t r) {
    const int64_t i = rows ? rows[r] : r;
    pack_row(s, i, r, mx, threats.data() + (size_t)r * CNNUE_AZ_THREAT_MAX, dims[r].threats, out);
  });
  return CNNUE_OK;
}

}  // extern "C"

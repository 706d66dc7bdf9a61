// Model files in the reference's text format (src/mojotrees/serialize.mojo):
// a whitespace-separated token stream, every float written as the decimal
// value of its IEEE-754 bit pattern, so a save/load round trip is bit-exact.
//
// Writer: format v4 (serialize.mojo:999-1119 save_model /
// save_multiclass_model, :431-446 mapper, :485-543 trees, :545-572
// categorical).  Reader: v1-v4 (serialize.mojo:1121-1370, 1463-1580).  v5
// files carry linear leaves, CTR tables or a narrowed feature pool, none of
// which this library trains or predicts with, and are refused by name.
#include <stdint.h>
#include <string.h>

#include <cmath>
#include <cstdio>
#include <algorithm>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "model.h"
#include "trainer.h"

namespace mtb {
namespace {

constexpr int kCatWords = 4;  // 256-bit category sets (categorical.mojo:115)

std::string f64_token(double x) {
  uint64_t b;
  memcpy(&b, &x, 8);
  return std::to_string(b);
}

// A tree as the format lays it out, from this library's node records.
struct TreeArrays {
  std::vector<long long> feature, thr, left, right, dleft, mbin, cat_off;
  std::vector<double> value, gain, count;
  std::vector<uint64_t> pool;
  int n_leaves = 0;
};

TreeArrays to_arrays(const std::vector<HostNode>& t) {
  TreeArrays a;
  for (const HostNode& nd : t) {
    const bool leaf = nd.feature < 0;
    a.n_leaves += leaf ? 1 : 0;
    a.feature.push_back(leaf ? -1 : nd.feature);
    a.left.push_back(leaf ? -1 : nd.left);
    a.right.push_back(leaf ? -1 : nd.right);
    a.value.push_back(nd.value);
    a.gain.push_back(leaf ? 0.0 : nd.gain);
    a.count.push_back((double)nd.count);
    // tree.mojo:461-480: a categorical node routes by its set alone
    if (!leaf && nd.is_cat) {
      a.thr.push_back(-1);
      a.dleft.push_back(0);
      a.mbin.push_back(-1);
      a.cat_off.push_back((long long)a.pool.size());
      for (int w = 0; w < kCatWords; ++w) a.pool.push_back(nd.bits[w]);
    } else {
      a.thr.push_back(leaf ? -1 : nd.thr);
      a.dleft.push_back(!leaf && nd.dleft ? 1 : 0);
      a.mbin.push_back(leaf ? -1 : nd.mbin);
      a.cat_off.push_back(-1);
    }
  }
  return a;
}

template <typename T>
void write_row(std::ostream& os, const std::vector<T>& v) {
  for (const T& x : v) os << x << ' ';
  os << '\n';
}

void write_f64_row(std::ostream& os, const std::vector<double>& v) {
  for (double x : v) os << f64_token(x) << ' ';
  os << '\n';
}

}  // namespace

void save_model_v4(const Model& m, std::ostream& os) {
  const BinMapper& mp = m.mapper;
  if (mp.n_features != m.n_features || (int64_t)mp.edge_offsets.size() != (int64_t)m.n_features + 1)
    throw std::runtime_error("model has no bin mapper to write");
  os << "mojotrees v4\n";
  if (m.objective == OBJECTIVE_MULTICLASS) {
    os << "multiclass " << m.num_class << '\n';
    os << "learning_rate " << f64_token(m.learning_rate) << '\n';
    os << "base_scores";
    for (int k = 0; k < m.num_class; ++k) os << ' ' << f64_token(m.base_scores[k]);
    os << '\n';
  } else {
    os << "objective " << m.objective << '\n';
    os << "learning_rate " << f64_token(m.learning_rate) << '\n';
    os << "base_score " << f64_token(m.base_scores[0]) << '\n';
  }
  // mapper: header, edges, offsets, per-feature missing bins
  os << "mapper " << mp.n_features << ' ' << mp.n_bins << ' ' << mp.edges.size() << '\n';
  write_f64_row(os, mp.edges);
  write_row(os, mp.edge_offsets);
  write_row(os, mp.missing_bin);
  // categorical tables, only when a feature is categorical
  bool any_cat = false;
  for (uint8_t c : mp.is_cat) any_cat = any_cat || c;
  if (any_cat) {
    os << "categorical " << mp.n_features << ' ' << mp.cat_codes.size() << '\n';
    for (int f = 0; f < mp.n_features; ++f) os << (mp.is_cat[f] ? 1 : 0) << ' ';
    os << '\n';
    write_row(os, mp.cat_codes);
    if (mp.cat_offsets.empty()) {
      for (int f = 0; f <= mp.n_features; ++f) os << "0 ";
      os << '\n';
    } else {
      write_row(os, mp.cat_offsets);
    }
  }
  os << "trees " << m.trees.size() << '\n';
  for (const auto& t : m.trees) {
    const TreeArrays a = to_arrays(t);
    os << "tree " << t.size() << ' ' << a.n_leaves << '\n';
    write_row(os, a.feature);
    write_row(os, a.thr);
    write_row(os, a.left);
    write_row(os, a.right);
    write_f64_row(os, a.value);
    write_row(os, a.dleft);
    write_row(os, a.mbin);
    bool covers = !a.count.empty();
    for (double c : a.count) covers = covers && c > 0.0;
    os << "counts " << (covers ? 1 : 0) << '\n';
    if (covers) write_f64_row(os, a.count);
    bool gains = false;
    for (double g : a.gain) gains = gains || g > 0.0;
    os << "gains " << (gains ? 1 : 0) << '\n';
    if (gains) write_f64_row(os, a.gain);
    if (!a.pool.empty()) {
      os << "cat " << a.pool.size() << '\n';
      write_row(os, a.cat_off);
      write_row(os, a.pool);
    }
  }
}

namespace {

struct Tokens {
  std::vector<std::string> t;
  size_t pos = 0;
  explicit Tokens(const std::string& content) {
    std::istringstream is(content);
    std::string s;
    while (is >> s) t.push_back(s);
  }
  const std::string& next() {
    if (pos >= t.size()) throw std::runtime_error("unexpected end of model file");
    return t[pos++];
  }
  std::string peek() const { return pos < t.size() ? t[pos] : std::string(); }
  size_t left() const { return t.size() - pos; }
  // a count the rest of the file must hold at least per_item tokens for;
  // checked before anything is sized by it
  void need(long long count, long long per_item) const {
    if (count < 0 || (per_item > 0 && (unsigned long long)count > left() / (unsigned long long)per_item))
      throw std::runtime_error("corrupt model file: a count exceeds what the file holds");
  }
  void expect(const char* tag) {
    if (next() != tag) throw std::runtime_error(std::string("corrupt model file: expected '") + tag + "'");
  }
  long long next_int() {
    const std::string& s = next();
    size_t i = 0;
    bool neg = false;
    if (!s.empty() && s[0] == '-') {
      neg = true;
      i = 1;
    }
    if (i >= s.size()) throw std::runtime_error("corrupt model file: empty integer token");
    unsigned long long v = 0;
    for (; i < s.size(); ++i) {
      if (s[i] < '0' || s[i] > '9') throw std::runtime_error("corrupt model file: invalid integer token '" + s + "'");
      const unsigned long long d = (unsigned long long)(s[i] - '0');
      if (v > (9223372036854775807ull - d) / 10) throw std::runtime_error("corrupt model file: integer out of range");
      v = v * 10 + d;
    }
    return neg ? -(long long)v : (long long)v;
  }
  // serialize.mojo:218-242: the whole u64 range, exactly
  uint64_t next_u64() {
    const std::string& s = next();
    if (s.empty()) throw std::runtime_error("corrupt model file: empty integer token");
    uint64_t v = 0;
    for (char c : s) {
      if (c < '0' || c > '9') throw std::runtime_error("corrupt model file: invalid digit in '" + s + "'");
      const uint64_t d = (uint64_t)(c - '0');
      if (v > (~0ull - d) / 10) throw std::runtime_error("corrupt model file: integer token does not fit in 64 bits");
      v = v * 10 + d;
    }
    return v;
  }
  double next_f64() {
    const uint64_t b = next_u64();
    double x;
    memcpy(&x, &b, 8);
    return x;
  }
};

// validation.mojo:1308+ check_tree_topology: internal nodes have two
// distinct children after them, leaves none, every node but the root is a
// child exactly once, the leaf count matches the header.
void check_topology(const std::vector<HostNode>& t, long long n_leaves, int n_features) {
  const long long n = (long long)t.size();
  std::vector<int> parents((size_t)n, 0);
  long long leaves = 0;
  for (long long i = 0; i < n; ++i) {
    const HostNode& nd = t[(size_t)i];
    if (nd.feature >= n_features) throw std::runtime_error("corrupt tree: split feature out of range");
    if (nd.feature < 0) {
      ++leaves;
      continue;
    }
    if (nd.left <= i || nd.right <= i || nd.left >= n || nd.right >= n || nd.left == nd.right)
      throw std::runtime_error("corrupt tree: child index out of order or out of range");
    ++parents[(size_t)nd.left];
    ++parents[(size_t)nd.right];
  }
  if (n > 0 && parents[0] != 0) throw std::runtime_error("corrupt tree: the root is some node's child");
  for (long long i = 1; i < n; ++i)
    if (parents[(size_t)i] != 1) throw std::runtime_error("corrupt tree: a node is not a child exactly once");
  if (leaves != n_leaves) throw std::runtime_error("corrupt tree: leaf count does not match the header");
}

}  // namespace

Model load_model_text(const std::string& content) {
  Tokens r(content);
  if (r.next() != "mojotrees") throw std::runtime_error("not a mojotrees model file");
  const std::string ver = r.next();
  int version;
  if (ver == "v1") version = 1;
  else if (ver == "v2") version = 2;
  else if (ver == "v3") version = 3;
  else if (ver == "v4") version = 4;
  else if (ver == "v5")
    throw Unsupported("format v5 model files (linear leaves, CTR tables or a narrowed feature pool) are not "
                      "covered by this library");
  else
    throw std::runtime_error("unsupported model format version '" + ver + "'");
  if (r.peek() == "feature_names") {  // names are not part of a model here
    r.next();
    const long long n = r.next_int();
    if (n < 1) throw std::runtime_error("corrupt feature_names section");
    r.need(n, 1);
    for (long long i = 0; i < n; ++i) r.next();
  }
  Model m;
  const std::string kind = r.next();
  if (kind == "objective") {
    const long long obj = r.next_int();
    if (obj != OBJECTIVE_L2 && obj != OBJECTIVE_BINARY)
      throw Unsupported("objective code " + std::to_string(obj) + " is not covered by this library");
    m.objective = (int)obj;
    m.num_class = 1;
    r.expect("learning_rate");
    m.learning_rate = r.next_f64();
    r.expect("base_score");
    m.base_scores = {r.next_f64()};
  } else if (kind == "multiclass") {
    const long long k = r.next_int();
    if (k < 2 || k > 1000000) throw std::runtime_error("corrupt model file: n_classes must be at least 2");
    m.objective = OBJECTIVE_MULTICLASS;
    m.num_class = (int)k;
    r.expect("learning_rate");
    m.learning_rate = r.next_f64();
    r.expect("base_scores");
    r.need(k, 1);
    for (long long i = 0; i < k; ++i) m.base_scores.push_back(r.next_f64());
  } else {
    throw std::runtime_error("corrupt model file: unknown model kind");
  }
  // mapper (serialize.mojo:1121-1194)
  BinMapper& mp = m.mapper;
  r.expect("mapper");
  const long long nf = r.next_int(), nb = r.next_int(), ne = r.next_int();
  if (nf < 1 || nf > (1ll << 24) || ne < 0 || ne > (1ll << 32)) throw std::runtime_error("corrupt mapper header");
  r.need(ne + nf + 1, 1);
  if (nb < 1 || nb > 256) throw std::runtime_error("corrupt mapper: n_bins must be in [1, 256]");
  mp.n_features = (int)nf;
  mp.n_bins = (int)nb;
  mp.edges.resize((size_t)ne);
  for (auto& e : mp.edges) e = r.next_f64();
  mp.edge_offsets.resize((size_t)nf + 1);
  for (auto& o : mp.edge_offsets) o = r.next_int();
  if (mp.edge_offsets[0] != 0 || mp.edge_offsets[(size_t)nf] != ne) throw std::runtime_error("corrupt mapper offsets");
  for (long long f = 0; f < nf; ++f) {
    const long long w = mp.edge_offsets[(size_t)f + 1] - mp.edge_offsets[(size_t)f];
    if (w < 0 || w > nb - 1) throw std::runtime_error("corrupt mapper offsets");
  }
  mp.missing_bin.assign((size_t)nf, -1);
  if (version >= 2)
    for (auto& v : mp.missing_bin) {
      const long long b = r.next_int();
      if (b < -1 || b >= nb) throw std::runtime_error("corrupt mapper: missing bin out of range");
      v = (int)b;
    }
  mp.is_cat.assign((size_t)nf, 0);
  mp.cat_offsets.assign((size_t)nf + 1, 0);
  if (r.peek() == "categorical") {
    r.next();
    const long long n_flags = r.next_int(), n_codes = r.next_int();
    if (n_flags != nf || n_codes < 0 || n_codes > (1ll << 32)) throw std::runtime_error("corrupt categorical header");
    r.need(nf + n_codes + nf + 1, 1);
    for (auto& c : mp.is_cat) c = r.next_int() != 0 ? 1 : 0;
    mp.cat_codes.resize((size_t)n_codes);
    for (auto& c : mp.cat_codes) c = r.next_int();
    for (auto& o : mp.cat_offsets) o = r.next_int();
    if (mp.cat_offsets[0] != 0 || mp.cat_offsets[(size_t)nf] != n_codes)
      throw std::runtime_error("corrupt categorical offsets");
    for (long long f = 0; f < nf; ++f) {
      const long long a = mp.cat_offsets[(size_t)f], b = mp.cat_offsets[(size_t)f + 1];
      if (b < a || b - a >= nb) throw std::runtime_error("corrupt categorical offsets");
      if (b > a && !mp.is_cat[(size_t)f]) throw std::runtime_error("corrupt categorical: table on a numerical feature");
      for (long long i = a + 1; i < b; ++i)
        if (mp.cat_codes[(size_t)i] <= mp.cat_codes[(size_t)i - 1])
          throw std::runtime_error("corrupt categorical: codes are not ascending");
    }
  }
  if (r.peek() == "monotone") {  // constraints bind training only; prediction ignores them
    r.next();
    const long long n = r.next_int();
    if (n != nf) throw std::runtime_error("corrupt model file: monotone section size");
    for (long long i = 0; i < n; ++i) r.next_int();
  }
  m.n_features = (int)nf;
  // trees (serialize.mojo:1235-1370)
  r.expect("trees");
  const long long n_trees = r.next_int();
  if (n_trees < 0 || n_trees > (1ll << 24)) throw std::runtime_error("corrupt model file: tree count");
  if (n_trees % m.num_class != 0) throw std::runtime_error("corrupt model file: tree count not divisible by classes");
  r.need(n_trees, 3);  // "tree", node count, leaf count at least
  bool mapper_fits = true;  // every split is one this mapper's bins can express
  m.trees.resize((size_t)n_trees);
  for (auto& t : m.trees) {
    r.expect("tree");
    const long long nn = r.next_int(), n_leaves = r.next_int();
    if (nn < 1 || nn > (1ll << 24) || n_leaves < 1 || n_leaves > nn) throw std::runtime_error("corrupt tree header");
    r.need(nn, version >= 2 ? 7 : 5);  // the per-node rows that always follow
    t.assign((size_t)nn, HostNode{});
    for (auto& nd : t) nd.feature = (int)r.next_int();
    for (auto& nd : t) nd.thr = (int)r.next_int();
    for (auto& nd : t) nd.left = (int)r.next_int();
    for (auto& nd : t) nd.right = (int)r.next_int();
    for (auto& nd : t) nd.value = r.next_f64();
    if (version >= 2) {
      for (auto& nd : t) nd.dleft = r.next_int() != 0 ? 1 : 0;
      for (auto& nd : t) {
        const long long b = r.next_int();
        if (b < -1 || b >= nb) throw std::runtime_error("corrupt tree: missing bin out of range");
        nd.mbin = (int)b;
      }
    } else {
      for (auto& nd : t) nd.mbin = -1;
    }
    bool has_counts = version == 3;
    if (version >= 4) {
      r.expect("counts");
      has_counts = r.next_int() != 0;
    }
    if (has_counts)
      for (auto& nd : t) {
        const double c = r.next_f64();
        if (!(c >= 0.0) || !(c < 9.0e18)) throw std::runtime_error("corrupt tree: node cover out of range");
        nd.count = (long long)c;
      }
    if (version >= 4) {
      r.expect("gains");
      if (r.next_int() != 0)
        for (auto& nd : t) {
          nd.gain = r.next_f64();
          if (nd.gain != nd.gain) throw std::runtime_error("corrupt tree: split gain is NaN");
        }
    }
    if (version >= 2 && r.peek() == "cat") {
      r.next();
      const long long nw = r.next_int();
      if (nw < 0 || nw % kCatWords != 0 || nw > (1ll << 30)) throw std::runtime_error("corrupt tree: category bitset size");
      r.need(nn + nw, 1);
      std::vector<long long> off((size_t)nn);
      for (auto& o : off) {
        o = r.next_int();
        if (o < -1 || o > nw - kCatWords || (o >= 0 && o % kCatWords != 0))
          throw std::runtime_error("corrupt tree: category set offset");
      }
      std::vector<uint64_t> pool((size_t)nw);
      for (auto& w : pool) w = r.next_u64();
      for (long long i = 0; i < nn; ++i)
        if (off[(size_t)i] >= 0 && t[(size_t)i].feature >= 0) {
          HostNode& nd = t[(size_t)i];
          nd.is_cat = 1;
          for (int w = 0; w < kCatWords; ++w) nd.bits[w] = pool[(size_t)off[(size_t)i] + w];
        }
    }
    check_topology(t, n_leaves, (int)nf);
    for (const auto& nd : t) {
      if (nd.feature < 0) continue;
      const long long k = mp.edge_offsets[(size_t)nd.feature + 1] - mp.edge_offsets[(size_t)nd.feature];
      if (nd.is_cat ? !mp.is_cat[(size_t)nd.feature] : nd.thr > k) mapper_fits = false;
    }
  }
  // A model trained on pre-binned columns is written with an edge-free
  // mapper; its splits then name bins that mapper cannot produce, and
  // raw-value prediction of it is refused rather than answered wrongly.
  m.has_mapper = mapper_fits;
  return m;
}

// ---------------------------------------------------------------------------
// The reference's inspection dump (src/mojotrees/model_dump.mojo :99-760,
// written as JSON by inspection.mojo :78-330): the model, its binning and
// every node, with thresholds as raw values and category sets as codes.
// Numbers are written to round-trip exactly ("%.17g"); NaN and infinities
// become null.
// ---------------------------------------------------------------------------
namespace {

std::string jnum(double x) {
  if (!std::isfinite(x)) return "null";
  char buf[40];
  snprintf(buf, sizeof buf, "%.17g", x);
  return buf;
}

struct DumpCtx {
  const Model& m;
  bool has_gain;
  std::vector<std::string> names;
};

void dump_node(std::string& out, const DumpCtx& c, const std::vector<HostNode>& t, const std::vector<int>& depth,
               const std::vector<int>& leaf_ord, const std::vector<int>& split_ord, int node) {
  const HostNode& nd = t[(size_t)node];
  const BinMapper& mp = c.m.mapper;
  out += "{\"node_index\":" + std::to_string(node);
  if (nd.feature < 0) {
    out += ",\"leaf_index\":" + std::to_string(leaf_ord[(size_t)node]);
    out += ",\"leaf_value\":" + jnum(nd.value) + ",\"leaf_count\":" + jnum((double)nd.count);
    out += ",\"depth\":" + std::to_string(depth[(size_t)node]) + "}";
    return;
  }
  const int f = nd.feature;
  out += ",\"split_index\":" + std::to_string(split_ord[(size_t)node]);
  out += ",\"split_feature\":" + std::to_string(f) + ",\"split_feature_name\":\"" + c.names[(size_t)f] + "\"";
  out += std::string(",\"decision_type\":") + (nd.is_cat ? "\"==\"" : "\"<=\"");
  // threshold_value (model_dump.mojo:456-486): the split bin's upper edge
  const bool feature_cat = f < (int)mp.is_cat.size() && mp.is_cat[(size_t)f];
  const long long e0 = mp.edge_offsets[(size_t)f], e1 = mp.edge_offsets[(size_t)f + 1];
  const bool has_thr = !nd.is_cat && !feature_cat && nd.thr >= 0 && nd.thr < e1 - e0;
  out += ",\"threshold\":" + (has_thr ? jnum(mp.edges[(size_t)(e0 + nd.thr)]) : std::string("null"));
  out += ",\"threshold_bin\":" + std::to_string(nd.is_cat ? -1 : nd.thr);
  if (nd.is_cat) {
    // category_bins / category_codes (model_dump.mojo:410-453)
    std::string bins = "[", codes = "[";
    const long long c0 = mp.cat_offsets.empty() ? 0 : mp.cat_offsets[(size_t)f];
    const long long nc = mp.n_categories(f);
    bool first = true;
    for (int b = 0; b < 256; ++b)
      if ((nd.bits[b >> 6] >> (b & 63)) & 1ull) {
        if (b < 1 || b > nc) throw std::runtime_error("dump: a category set names a bin with no category");
        bins += (first ? "" : ",") + std::to_string(b);
        codes += (first ? "" : ",") + std::to_string(mp.cat_codes[(size_t)(c0 + b - 1)]);
        first = false;
      }
    out += ",\"categories\":" + codes + "],\"category_bins\":" + bins + "]";
  } else {
    out += ",\"categories\":null,\"category_bins\":null";
  }
  const int mb = nd.is_cat ? -1 : nd.mbin;
  out += std::string(",\"default_left\":") + (!nd.is_cat && nd.dleft ? "true" : "false");
  out += ",\"missing_bin\":" + std::to_string(mb);
  out += std::string(",\"missing_type\":") + (mb >= 0 ? "\"NaN\"" : "\"None\"");
  out += ",\"split_gain\":" + (c.has_gain ? jnum(nd.gain) : std::string("null"));
  out += ",\"internal_value\":" + jnum(nd.value) + ",\"internal_count\":" + jnum((double)nd.count);
  out += ",\"depth\":" + std::to_string(depth[(size_t)node]);
  out += ",\"left_child\":";
  dump_node(out, c, t, depth, leaf_ord, split_ord, nd.left);
  out += ",\"right_child\":";
  dump_node(out, c, t, depth, leaf_ord, split_ord, nd.right);
  out += "}";
}

}  // namespace

std::string dump_model_json(const Model& m) {
  const BinMapper& mp = m.mapper;
  const int K = m.num_class, F = m.n_features;
  if ((int64_t)mp.edge_offsets.size() != (int64_t)F + 1) throw std::runtime_error("model has no bin mapper to dump");
  DumpCtx c{m, false, {}};
  bool has_count = !m.trees.empty();
  for (const auto& t : m.trees)
    for (const auto& nd : t) {
      if (nd.feature >= 0 && nd.gain > 0.0) c.has_gain = true;
      if (!(nd.count > 0)) has_count = false;
    }
  for (int f = 0; f < F; ++f) c.names.push_back("Column_" + std::to_string(f));
  std::string out = "{\"dump_format_version\":1,\"producer\":\"mojotrees\",\"model_format_version\":4";
  out += ",\"source\":\"native\",\"objective_code\":";
  out += m.objective == OBJECTIVE_MULTICLASS ? std::string("null") : std::to_string(m.objective);
  out += ",\"num_class\":" + std::to_string(K) + ",\"num_tree_per_iteration\":" + std::to_string(K);
  out += ",\"num_iteration\":" + std::to_string(m.trees.size() / (size_t)K);
  out += ",\"learning_rate\":" + jnum(m.learning_rate) + ",\"base_score\":[";
  for (int k = 0; k < K; ++k) out += (k ? "," : "") + jnum(m.base_scores[(size_t)k]);
  out += "],\"leaf_value_is_shrunk\":false,\"num_feature\":" + std::to_string(F);
  out += ",\"max_feature_idx\":" + std::to_string(F - 1) + ",\"num_bin\":" + std::to_string(mp.n_bins);
  out += ",\"feature_names\":[";
  for (int f = 0; f < F; ++f) out += (f ? ",\"" : "\"") + c.names[(size_t)f] + "\"";
  out += "],\"feature_infos\":[";
  for (int f = 0; f < F; ++f) {
    const bool cat = f < (int)mp.is_cat.size() && mp.is_cat[(size_t)f];
    const int mb = mp.missing_bin[(size_t)f];
    out += (f ? ",{" : "{") + std::string("\"index\":") + std::to_string(f) + ",\"name\":\"" + c.names[(size_t)f] + "\"";
    out += ",\"missing_bin\":" + std::to_string(mb) + std::string(",\"missing_type\":") + (mb >= 0 ? "\"NaN\"" : "\"None\"");
    out += ",\"monotone\":0";
    if (cat) {
      const long long c0 = mp.cat_offsets[(size_t)f], nc = mp.n_categories(f);
      out += ",\"type\":\"categorical\",\"categories\":[";
      for (long long i = 0; i < nc; ++i) out += (i ? "," : "") + std::to_string(mp.cat_codes[(size_t)(c0 + i)]);
      out += "],\"bin_upper_bounds\":null,\"num_bin\":" + std::to_string(nc + 1) + "}";
    } else {
      const long long e0 = mp.edge_offsets[(size_t)f], e1 = mp.edge_offsets[(size_t)f + 1];
      out += ",\"type\":\"numerical\",\"categories\":null,\"bin_upper_bounds\":[";
      for (long long i = e0; i < e1; ++i) out += (i > e0 ? "," : "") + jnum(mp.edges[(size_t)i]);
      out += "],\"num_bin\":" + std::to_string(e1 - e0 + 1 + (mb >= 0 ? 1 : 0)) + "}";
    }
  }
  out += "],\"monotone_constraints\":null";
  out += std::string(",\"has_split_gain\":") + (c.has_gain ? "true" : "false");
  out += std::string(",\"has_node_count\":") + (has_count ? "true" : "false");
  out += ",\"linear_tree\":false,\"tree_info\":[";
  for (size_t ti = 0; ti < m.trees.size(); ++ti) {
    const auto& t = m.trees[ti];
    const size_t n = t.size();
    std::vector<int> depth(n, 0), leaf_ord(n, -1), split_ord(n, -1);
    int leaves = 0, splits = 0, n_cat = 0, max_depth = 0;
    for (size_t i = 0; i < n; ++i) {
      if (t[i].feature < 0) {
        leaf_ord[i] = leaves++;
        continue;
      }
      split_ord[i] = splits++;
      n_cat += t[i].is_cat ? 1 : 0;
      depth[(size_t)t[i].left] = depth[i] + 1;  // children follow their parent in node order
      depth[(size_t)t[i].right] = depth[i] + 1;
    }
    for (size_t i = 0; i < n; ++i) max_depth = std::max(max_depth, depth[i]);
    out += (ti ? ",{" : "{") + std::string("\"tree_index\":") + std::to_string(ti);
    out += ",\"iteration\":" + std::to_string(ti / (size_t)K) + ",\"class_id\":" + std::to_string(ti % (size_t)K);
    out += ",\"num_leaves\":" + std::to_string(leaves) + ",\"num_nodes\":" + std::to_string(n);
    out += ",\"num_cat\":" + std::to_string(n_cat) + ",\"max_depth\":" + std::to_string(max_depth);
    out += ",\"shrinkage\":" + jnum(m.learning_rate) + ",\"tree_structure\":";
    if (n) dump_node(out, c, t, depth, leaf_ord, split_ord, 0);
    else out += "null";
    out += "}";
  }
  out += "]}";
  return out;
}

}  // namespace mtb

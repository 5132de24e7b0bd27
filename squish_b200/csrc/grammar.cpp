// grammar.cpp — JSON-constrained decoding on the host: a byte-level JSON pushdown matcher and
// the per-step token bitmask it allows, for the fused sampler's grammar mask (sampler.cu).
//
// The reference builds token bitmasks with xgrammar (squish/grammar/grammar_engine.py:220-254)
// and a character FSM for schemas (squish/grammar/schema_gen.py:172-330). Here:
//   VocabIndex   the tokenizer's byte strings in a trie (built once per tokenizer), plus the
//                set of "plain string" tokens (no '"', '\\' or control bytes), which are
//                allowed whenever the matcher is inside a JSON string, whatever the stack.
//   JsonMatcher  a fixed-size POD state (container stack of up to 64 frames, lexer state,
//                literal progress, whitespace run) with step(byte) -> accepted?. allowed_mask
//                walks the trie depth first, copying the state per node and pruning a subtree at
//                the first rejected byte; inside a string it starts from the plain-string set and
//                walks only the trie of the other tokens. EOS is allowed once the top-level
//                value is complete; runs of whitespace are capped so a model cannot pad forever.
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace sqgram {

namespace {

constexpr int kMaxDepth = 64;

enum Lex : uint8_t {
  L_STRUCT,  // between tokens: expectations come from the top frame (or the top level)
  L_STR, L_ESC, L_U1, L_U2, L_U3, L_U4,
  L_NUM_MINUS, L_NUM_ZERO, L_NUM_INT, L_NUM_DOT, L_NUM_FRAC, L_NUM_E, L_NUM_ESIGN, L_NUM_EXP,
  L_LIT,
};

enum Frame : uint8_t {
  F_OBJ_KEY_OR_END, F_OBJ_KEY, F_OBJ_COLON, F_OBJ_VALUE, F_OBJ_AFTER,
  F_ARR_VALUE_OR_END, F_ARR_VALUE, F_ARR_AFTER,
};

const char* const kLits[3] = {"true", "false", "null"};
const uint8_t kLitLen[3] = {4, 5, 4};

inline bool is_ws(uint8_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
inline bool is_digit(uint8_t c) { return c >= '0' && c <= '9'; }
inline bool is_hex(uint8_t c) { return is_digit(c) || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F'); }

struct State {
  uint8_t stack[kMaxDepth];
  int8_t depth = 0;
  uint8_t lex = L_STRUCT;
  uint8_t lit = 0, lit_pos = 0;
  uint8_t key = 0;      // the current string is an object key
  uint8_t done = 0;     // the top-level value is complete
  uint8_t ws_run = 0;   // consecutive whitespace bytes
  uint8_t top_object = 1;  // the top-level value must be an object
  uint8_t max_ws = 24;
};

inline void value_done(State& s) {
  s.lex = L_STRUCT;
  if (s.depth == 0) {
    s.done = 1;
    return;
  }
  uint8_t& f = s.stack[s.depth - 1];
  if (f == F_OBJ_VALUE) f = F_OBJ_AFTER;
  else f = F_ARR_AFTER;  // F_ARR_VALUE or F_ARR_VALUE_OR_END
}

inline bool start_value(State& s, uint8_t c) {
  if (s.depth == 0 && s.top_object && c != '{') return false;
  switch (c) {
    case '{':
      if (s.depth >= kMaxDepth) return false;
      s.stack[s.depth++] = F_OBJ_KEY_OR_END;
      return true;
    case '[':
      if (s.depth >= kMaxDepth) return false;
      s.stack[s.depth++] = F_ARR_VALUE_OR_END;
      return true;
    case '"': s.lex = L_STR; s.key = 0; return true;
    case '-': s.lex = L_NUM_MINUS; return true;
    case '0': s.lex = L_NUM_ZERO; return true;
    case 't': s.lex = L_LIT; s.lit = 0; s.lit_pos = 1; return true;
    case 'f': s.lex = L_LIT; s.lit = 1; s.lit_pos = 1; return true;
    case 'n': s.lex = L_LIT; s.lit = 2; s.lit_pos = 1; return true;
    default:
      if (c >= '1' && c <= '9') { s.lex = L_NUM_INT; return true; }
      return false;
  }
}

inline bool close(State& s, uint8_t c) {
  const uint8_t f = s.stack[s.depth - 1];
  const bool obj = f <= F_OBJ_AFTER;
  if (obj ? c != '}' : c != ']') return false;
  --s.depth;
  value_done(s);
  return true;
}

bool step_struct(State& s, uint8_t c) {
  if (is_ws(c)) {
    if (s.ws_run >= s.max_ws) return false;
    ++s.ws_run;
    return true;
  }
  s.ws_run = 0;
  if (s.depth == 0) return s.done ? false : start_value(s, c);
  uint8_t& f = s.stack[s.depth - 1];
  switch (f) {
    case F_OBJ_KEY_OR_END:
      if (c == '}') return close(s, c);
      [[fallthrough]];
    case F_OBJ_KEY:
      if (c != '"') return false;
      s.lex = L_STR;
      s.key = 1;
      return true;
    case F_OBJ_COLON:
      if (c != ':') return false;
      f = F_OBJ_VALUE;
      return true;
    case F_OBJ_VALUE:
    case F_ARR_VALUE:
      return start_value(s, c);
    case F_ARR_VALUE_OR_END:
      if (c == ']') return close(s, c);
      return start_value(s, c);
    case F_OBJ_AFTER:
      if (c == ',') { f = F_OBJ_KEY; return true; }
      return close(s, c);
    case F_ARR_AFTER:
      if (c == ',') { f = F_ARR_VALUE; return true; }
      return close(s, c);
  }
  return false;
}

// a number ends at the first byte that cannot continue it; that byte is then read structurally
inline bool end_number(State& s, uint8_t c) {
  value_done(s);
  return step_struct(s, c);
}

bool step(State& s, uint8_t c) {
  switch (s.lex) {
    case L_STRUCT: return step_struct(s, c);
    case L_STR:
      if (c == '"') {
        if (s.key) {
          s.lex = L_STRUCT;
          s.stack[s.depth - 1] = F_OBJ_COLON;
        } else {
          value_done(s);
        }
        return true;
      }
      if (c == '\\') { s.lex = L_ESC; return true; }
      return c >= 0x20;
    case L_ESC:
      if (c == 'u') { s.lex = L_U1; return true; }
      if (c == '"' || c == '\\' || c == '/' || c == 'b' || c == 'f' || c == 'n' || c == 'r' || c == 't') {
        s.lex = L_STR;
        return true;
      }
      return false;
    case L_U1: case L_U2: case L_U3: case L_U4:
      if (!is_hex(c)) return false;
      s.lex = s.lex == L_U4 ? (uint8_t)L_STR : (uint8_t)(s.lex + 1);
      return true;
    case L_NUM_MINUS:
      if (c == '0') { s.lex = L_NUM_ZERO; return true; }
      if (c >= '1' && c <= '9') { s.lex = L_NUM_INT; return true; }
      return false;
    case L_NUM_ZERO:
      if (c == '.') { s.lex = L_NUM_DOT; return true; }
      if (c == 'e' || c == 'E') { s.lex = L_NUM_E; return true; }
      if (is_digit(c)) return false;
      return end_number(s, c);
    case L_NUM_INT:
      if (is_digit(c)) return true;
      if (c == '.') { s.lex = L_NUM_DOT; return true; }
      if (c == 'e' || c == 'E') { s.lex = L_NUM_E; return true; }
      return end_number(s, c);
    case L_NUM_DOT:
      if (!is_digit(c)) return false;
      s.lex = L_NUM_FRAC;
      return true;
    case L_NUM_FRAC:
      if (is_digit(c)) return true;
      if (c == 'e' || c == 'E') { s.lex = L_NUM_E; return true; }
      return end_number(s, c);
    case L_NUM_E:
      if (c == '+' || c == '-') { s.lex = L_NUM_ESIGN; return true; }
      if (is_digit(c)) { s.lex = L_NUM_EXP; return true; }
      return false;
    case L_NUM_ESIGN:
      if (!is_digit(c)) return false;
      s.lex = L_NUM_EXP;
      return true;
    case L_NUM_EXP:
      if (is_digit(c)) return true;
      return end_number(s, c);
    case L_LIT:
      if (c != (uint8_t)kLits[s.lit][s.lit_pos]) return false;
      if (++s.lit_pos == kLitLen[s.lit]) value_done(s);
      return true;
  }
  return false;
}

inline bool complete(const State& s) {
  if (s.depth != 0) return false;
  if (s.done) return s.lex == L_STRUCT;
  // a bare top-level number ends at end of input
  return !s.top_object && (s.lex == L_NUM_ZERO || s.lex == L_NUM_INT || s.lex == L_NUM_FRAC || s.lex == L_NUM_EXP);
}

}  // namespace

class VocabIndex {
 public:
  struct Node {
    std::vector<std::pair<uint8_t, int>> kids;  // sorted by byte
    std::vector<int> ends;                      // token ids whose bytes end here
  };

  VocabIndex(std::vector<std::string> tok_bytes, int64_t eos)
      : toks_(std::move(tok_bytes)), vocab_((int)toks_.size()), eos_((int)eos) {
    const std::vector<std::string>& toks = toks_;
    full_.emplace_back();
    special_.emplace_back();
    plain_.assign((vocab_ + 31) / 32, 0u);
    for (int id = 0; id < vocab_; ++id) {
      const std::string& b = toks[id];
      if (b.empty()) continue;  // special / unprintable tokens are never allowed inside JSON
      bool plain = true;
      for (unsigned char c : b) plain = plain && c != '"' && c != '\\' && c >= 0x20;
      insert(full_, b, id);
      if (plain) plain_[id >> 5] |= 1u << (id & 31);
      else insert(special_, b, id);
    }
  }
  int vocab() const { return vocab_; }
  int eos() const { return eos_; }
  const std::vector<Node>& full() const { return full_; }
  const std::vector<Node>& special() const { return special_; }
  const std::vector<uint32_t>& plain() const { return plain_; }
  const std::string& bytes_of(int64_t id) const { return toks_[id]; }

 private:
  static void insert(std::vector<Node>& t, const std::string& b, int id) {
    int n = 0;
    for (unsigned char c : b) {
      auto& kids = t[n].kids;
      auto it = std::lower_bound(kids.begin(), kids.end(), std::make_pair((uint8_t)c, -1));
      if (it != kids.end() && it->first == c) {
        n = it->second;
      } else {
        const int child = (int)t.size();
        kids.insert(it, {(uint8_t)c, child});
        t.emplace_back();
        n = child;
      }
    }
    t[n].ends.push_back(id);
  }
  std::vector<std::string> toks_;
  int vocab_, eos_;
  std::vector<Node> full_, special_;
  std::vector<uint32_t> plain_;
};

class JsonMatcher {
 public:
  JsonMatcher(std::shared_ptr<VocabIndex> vi, bool top_object, int64_t max_ws) : vi_(std::move(vi)) {
    s_.top_object = top_object ? 1 : 0;
    s_.max_ws = (uint8_t)std::min<int64_t>(std::max<int64_t>(max_ws, 1), 255);
  }

  // feed one generated token; false (and no state change) if the grammar rejects it
  bool advance(int64_t tok) {
    if (tok == vi_->eos()) {
      if (!complete(s_)) return false;
      terminated_ = true;
      return true;
    }
    if (tok < 0 || tok >= (int64_t)vi_->vocab() || vi_->bytes_of(tok).empty()) return false;
    State t = s_;
    for (unsigned char c : vi_->bytes_of(tok))
      if (!step(t, c)) return false;
    s_ = t;
    return true;
  }

  bool is_complete() const { return complete(s_); }
  bool is_terminated() const { return terminated_ || (s_.done && s_.depth == 0 && s_.lex == L_STRUCT); }

  torch::Tensor allowed_mask() const {
    const int words = (vi_->vocab() + 31) / 32;
    auto out = torch::zeros({words}, torch::kInt32);
    uint32_t* m = reinterpret_cast<uint32_t*>(out.data_ptr<int32_t>());
    if (s_.lex == L_STR) {
      std::memcpy(m, vi_->plain().data(), sizeof(uint32_t) * words);
      walk(vi_->special(), 0, s_, m);
    } else {
      walk(vi_->full(), 0, s_, m);
    }
    const int e = vi_->eos();
    if (complete(s_) && e >= 0 && e < vi_->vocab()) m[e >> 5] |= 1u << (e & 31);
    return out;
  }

 private:
  static void walk(const std::vector<VocabIndex::Node>& t, int n, const State& s, uint32_t* m) {
    for (int id : t[n].ends) m[id >> 5] |= 1u << (id & 31);
    for (const auto& kc : t[n].kids) {
      State c = s;
      if (step(c, kc.first)) walk(t, kc.second, c, m);
    }
  }

  std::shared_ptr<VocabIndex> vi_;
  State s_;
  bool terminated_ = false;
};

// ------------------------------------------------------------------------ schema-guided
// A JSON schema subset compiled to a node table (by serving/grammar.py): object (listed
// properties only, each at most once, `required` enforced before '}'), array (items), string,
// integer, number, boolean, null, enum / const (serialized literals), and any (generic JSON).
// The stack keeps per frame the object's node, the node of the member value being read and the
// set of properties already used; depth is limited to 16.
enum Kind : uint8_t { K_ANY, K_OBJECT, K_ARRAY, K_STRING, K_INTEGER, K_NUMBER, K_BOOLEAN, K_NULL, K_ENUM, K_UNION };

struct SchemaNode {
  uint8_t kind = K_ANY;
  std::vector<std::string> names;  // object property names (raw key bytes)
  std::vector<int> props;          // their nodes
  uint64_t required = 0;
  int items = -1;                  // array items node (-1: any)
  std::vector<std::string> lits;   // enum literals, serialized JSON
  // K_UNION (type lists, anyOf / oneOf): the alternatives are the `props` nodes (names empty)
};

class Schema {
 public:
  Schema(const std::vector<int64_t>& kinds, const std::vector<std::vector<std::pair<pybind11::bytes, int64_t>>>& props,
         const std::vector<int64_t>& required, const std::vector<int64_t>& items,
         const std::vector<std::vector<pybind11::bytes>>& lits, int64_t root)
      : root_((int)root) {
    const size_t n = kinds.size();
    TORCH_CHECK(props.size() == n && required.size() == n && items.size() == n && lits.size() == n,
                "schema tables must have one entry per node");
    TORCH_CHECK(n >= 1 && n < 65535 && root >= 0 && (size_t)root < n, "bad schema root / size");
    nodes_.resize(n);
    for (size_t i = 0; i < n; ++i) {
      SchemaNode& d = nodes_[i];
      d.kind = (uint8_t)kinds[i];
      TORCH_CHECK(props[i].size() <= 64, "at most 64 properties per object");
      for (const auto& pr : props[i]) {
        d.names.push_back(std::string(pr.first));
        TORCH_CHECK(pr.second >= 0 && (size_t)pr.second < n, "property node out of range");
        d.props.push_back((int)pr.second);
      }
      d.required = (uint64_t)required[i];
      d.items = (int)items[i];
      TORCH_CHECK(lits[i].size() <= 64, "at most 64 enum values");
      for (const auto& l : lits[i]) d.lits.push_back(std::string(l));
    }
  }
  const SchemaNode& node(int i) const { return nodes_[i]; }
  int root() const { return root_; }

 private:
  std::vector<SchemaNode> nodes_;
  int root_;
};

namespace {

constexpr int kSDepth = 16;
constexpr uint16_t kAnyNode = 0xFFFF;  // generic JSON below this point
enum : uint8_t { L_SKEY = 32, L_ENUM = 33 };

struct SState {
  uint8_t f[kSDepth];
  uint16_t node[kSDepth];   // schema node of the container
  uint16_t vnode[kSDepth];  // object frames: node of the member value being read
  uint64_t used[kSDepth];   // object frames: properties already present
  uint64_t cand = 0;        // key / enum candidates
  int8_t depth = 0;
  uint8_t lex = L_STRUCT, lit = 0, lit_pos = 0, key = 0, done = 0, ws_run = 0, max_ws = 24;
  uint8_t cpos = 0, num_int = 0;
  uint16_t enode = 0;       // enum node being matched
};

inline const SchemaNode* sn(const Schema& sc, uint16_t id) { return id == kAnyNode ? nullptr : &sc.node(id); }

inline uint16_t expected(const Schema& sc, const SState& s) {
  if (s.depth == 0) return (uint16_t)sc.root();
  const uint8_t f = s.f[s.depth - 1];
  if (f <= F_OBJ_AFTER) return s.vnode[s.depth - 1];
  const SchemaNode* n = sn(sc, s.node[s.depth - 1]);
  return (n == nullptr || n->items < 0) ? kAnyNode : (uint16_t)n->items;
}

inline void s_value_done(SState& s) {
  s.lex = L_STRUCT;
  if (s.depth == 0) {
    s.done = 1;
    return;
  }
  uint8_t& f = s.f[s.depth - 1];
  f = f == F_OBJ_VALUE ? F_OBJ_AFTER : F_ARR_AFTER;
}

inline bool s_push(SState& s, uint8_t f, uint16_t node) {
  if (s.depth >= kSDepth) return false;
  s.f[s.depth] = f;
  s.node[s.depth] = node;
  s.vnode[s.depth] = kAnyNode;
  s.used[s.depth] = 0;
  ++s.depth;
  return true;
}

// can a value of node `id` start with byte c (unions: any alternative)?
bool s_can_start(const Schema& sc, uint16_t id, uint8_t c, int depth = 0) {
  const SchemaNode* n = sn(sc, id);
  const uint8_t k = n == nullptr ? K_ANY : n->kind;
  switch (k) {
    case K_OBJECT: return c == '{';
    case K_ARRAY: return c == '[';
    case K_STRING: return c == '"';
    case K_INTEGER:
    case K_NUMBER: return c == '-' || is_digit(c);
    case K_BOOLEAN: return c == 't' || c == 'f';
    case K_NULL: return c == 'n';
    case K_ENUM:
      for (const auto& l : n->lits)
        if (!l.empty() && (uint8_t)l[0] == c) return true;
      return false;
    case K_UNION:
      if (depth > 8) return false;
      for (int a : n->props)
        if (s_can_start(sc, (uint16_t)a, c, depth + 1)) return true;
      return false;
    default:
      return c == '{' || c == '[' || c == '"' || c == '-' || is_digit(c) || c == 't' || c == 'f' || c == 'n';
  }
}

bool s_start_as(const Schema& sc, SState& s, uint16_t id, uint8_t c, int depth = 0);

bool s_start_value(const Schema& sc, SState& s, uint8_t c) { return s_start_as(sc, s, expected(sc, s), c); }

// Start a value of node `id` with byte c. A union picks the one alternative that can start
// with c; when several can (two objects, integer and number, ...), the value is read as any
// JSON value (integer + number alone: as a number), which allows a superset of the union.
bool s_start_as(const Schema& sc, SState& s, uint16_t id, uint8_t c, int depth) {
  const SchemaNode* n = sn(sc, id);
  if (n != nullptr && n->kind == K_UNION) {
    if (depth > 8) return false;
    int pick = -1, count = 0;
    bool all_numeric = true;
    for (int a : n->props)
      if (s_can_start(sc, (uint16_t)a, c)) {
        ++count;
        pick = a;
        const uint8_t ak = sc.node(a).kind;
        all_numeric = all_numeric && (ak == K_INTEGER || ak == K_NUMBER);
      }
    if (count == 0) return false;
    if (count == 1) return s_start_as(sc, s, (uint16_t)pick, c, depth + 1);
    if (all_numeric) {
      for (int a : n->props)
        if (sc.node(a).kind == K_NUMBER) return s_start_as(sc, s, (uint16_t)a, c, depth + 1);
    }
    return s_start_as(sc, s, kAnyNode, c, depth + 1);
  }
  const uint8_t k = n == nullptr ? K_ANY : n->kind;
  s.num_int = k == K_INTEGER;
  switch (k) {
    case K_OBJECT: return c == '{' && s_push(s, F_OBJ_KEY_OR_END, id);
    case K_ARRAY: return c == '[' && s_push(s, F_ARR_VALUE_OR_END, id);
    case K_STRING:
      if (c != '"') return false;
      s.lex = L_STR;
      s.key = 0;
      return true;
    case K_INTEGER:
    case K_NUMBER:
      if (c == '-') { s.lex = L_NUM_MINUS; return true; }
      if (c == '0') { s.lex = L_NUM_ZERO; return true; }
      if (c >= '1' && c <= '9') { s.lex = L_NUM_INT; return true; }
      return false;
    case K_BOOLEAN:
      if (c == 't') { s.lex = L_LIT; s.lit = 0; s.lit_pos = 1; return true; }
      if (c == 'f') { s.lex = L_LIT; s.lit = 1; s.lit_pos = 1; return true; }
      return false;
    case K_NULL:
      if (c != 'n') return false;
      s.lex = L_LIT;
      s.lit = 2;
      s.lit_pos = 1;
      return true;
    case K_ENUM: {
      uint64_t m = 0;
      for (size_t i = 0; i < n->lits.size(); ++i)
        if (!n->lits[i].empty() && (uint8_t)n->lits[i][0] == c) m |= 1ull << i;
      if (!m) return false;
      s.lex = L_ENUM;
      s.enode = id;
      s.cand = m;
      s.cpos = 1;
      return true;
    }
    default:  // any JSON value; containers below it are generic
      switch (c) {
        case '{': return s_push(s, F_OBJ_KEY_OR_END, kAnyNode);
        case '[': return s_push(s, F_ARR_VALUE_OR_END, kAnyNode);
        case '"': s.lex = L_STR; s.key = 0; return true;
        case '-': s.lex = L_NUM_MINUS; return true;
        case '0': s.lex = L_NUM_ZERO; return true;
        case 't': s.lex = L_LIT; s.lit = 0; s.lit_pos = 1; return true;
        case 'f': s.lex = L_LIT; s.lit = 1; s.lit_pos = 1; return true;
        case 'n': s.lex = L_LIT; s.lit = 2; s.lit_pos = 1; return true;
        default:
          if (c >= '1' && c <= '9') { s.lex = L_NUM_INT; return true; }
          return false;
      }
  }
}

inline bool s_obj_can_close(const Schema& sc, const SState& s) {
  const SchemaNode* n = sn(sc, s.node[s.depth - 1]);
  return n == nullptr || (n->required & ~s.used[s.depth - 1]) == 0;
}

inline bool s_obj_has_free_key(const Schema& sc, const SState& s) {
  const SchemaNode* n = sn(sc, s.node[s.depth - 1]);
  if (n == nullptr) return true;
  const uint64_t all = n->names.size() >= 64 ? ~0ull : ((1ull << n->names.size()) - 1);
  return (all & ~s.used[s.depth - 1]) != 0;
}

bool s_close(const Schema& sc, SState& s, uint8_t c) {
  const bool obj = s.f[s.depth - 1] <= F_OBJ_AFTER;
  if (obj ? c != '}' : c != ']') return false;
  if (obj && !s_obj_can_close(sc, s)) return false;
  --s.depth;
  s_value_done(s);
  return true;
}

bool s_step_struct(const Schema& sc, SState& s, uint8_t c) {
  if (is_ws(c)) {
    if (s.ws_run >= s.max_ws) return false;
    ++s.ws_run;
    return true;
  }
  s.ws_run = 0;
  if (s.depth == 0) return s.done ? false : s_start_value(sc, s, c);
  uint8_t& f = s.f[s.depth - 1];
  switch (f) {
    case F_OBJ_KEY_OR_END:
      if (c == '}') return s_close(sc, s, c);
      [[fallthrough]];
    case F_OBJ_KEY: {
      if (c != '"') return false;
      const SchemaNode* n = sn(sc, s.node[s.depth - 1]);
      if (n == nullptr) {
        s.lex = L_STR;
        s.key = 1;
        return true;
      }
      const uint64_t all = n->names.size() >= 64 ? ~0ull : ((1ull << n->names.size()) - 1);
      s.cand = all & ~s.used[s.depth - 1];
      if (!s.cand) return false;
      s.lex = L_SKEY;
      s.cpos = 0;
      return true;
    }
    case F_OBJ_COLON:
      if (c != ':') return false;
      f = F_OBJ_VALUE;
      return true;
    case F_OBJ_VALUE:
    case F_ARR_VALUE:
      return s_start_value(sc, s, c);
    case F_ARR_VALUE_OR_END:
      if (c == ']') return s_close(sc, s, c);
      return s_start_value(sc, s, c);
    case F_OBJ_AFTER:
      if (c == ',') {
        if (!s_obj_has_free_key(sc, s)) return false;
        f = F_OBJ_KEY;
        return true;
      }
      return s_close(sc, s, c);
    case F_ARR_AFTER:
      if (c == ',') { f = F_ARR_VALUE; return true; }
      return s_close(sc, s, c);
  }
  return false;
}

inline bool s_end_number(const Schema& sc, SState& s, uint8_t c) {
  s_value_done(s);
  return s_step_struct(sc, s, c);
}

bool s_step(const Schema& sc, SState& s, uint8_t c) {
  switch (s.lex) {
    case L_STRUCT: return s_step_struct(sc, s, c);
    case L_SKEY: {
      const SchemaNode& n = sc.node(s.node[s.depth - 1]);
      if (c == '"') {
        for (size_t i = 0; i < n.names.size(); ++i)
          if (((s.cand >> i) & 1) && n.names[i].size() == s.cpos) {
            s.used[s.depth - 1] |= 1ull << i;
            s.vnode[s.depth - 1] = (uint16_t)n.props[i];
            s.f[s.depth - 1] = F_OBJ_COLON;
            s.lex = L_STRUCT;
            return true;
          }
        return false;
      }
      uint64_t m = 0;
      for (size_t i = 0; i < n.names.size(); ++i)
        if (((s.cand >> i) & 1) && s.cpos < n.names[i].size() && (uint8_t)n.names[i][s.cpos] == c) m |= 1ull << i;
      if (!m) return false;
      s.cand = m;
      ++s.cpos;
      return true;
    }
    case L_ENUM: {
      const SchemaNode& n = sc.node(s.enode);
      uint64_t m = 0;
      bool complete = false;
      for (size_t i = 0; i < n.lits.size(); ++i) {
        if (!((s.cand >> i) & 1)) continue;
        if (s.cpos < n.lits[i].size() && (uint8_t)n.lits[i][s.cpos] == c) m |= 1ull << i;
        if (n.lits[i].size() == s.cpos) complete = true;
      }
      if (m) {
        s.cand = m;
        ++s.cpos;
        // a quoted literal ends with its closing quote; other literals end at the next byte
        for (size_t i = 0; i < n.lits.size(); ++i)
          if (((m >> i) & 1) && n.lits[i].size() == s.cpos && n.lits[i].back() == '"') {
            bool longer = false;
            for (size_t j = 0; j < n.lits.size(); ++j) longer = longer || (((m >> j) & 1) && n.lits[j].size() > s.cpos);
            if (!longer) s_value_done(s);
            break;
          }
        return true;
      }
      if (!complete) return false;
      s_value_done(s);
      return s_step_struct(sc, s, c);
    }
    case L_STR:
      if (c == '"') {
        if (s.key) {
          s.lex = L_STRUCT;
          s.f[s.depth - 1] = F_OBJ_COLON;
          s.vnode[s.depth - 1] = kAnyNode;
        } else {
          s_value_done(s);
        }
        return true;
      }
      if (c == '\\') { s.lex = L_ESC; return true; }
      return c >= 0x20;
    case L_NUM_ZERO:
      if (s.num_int && (c == '.' || c == 'e' || c == 'E')) return false;
      if (c == '.') { s.lex = L_NUM_DOT; return true; }
      if (c == 'e' || c == 'E') { s.lex = L_NUM_E; return true; }
      if (is_digit(c)) return false;
      return s_end_number(sc, s, c);
    case L_NUM_INT:
      if (is_digit(c)) return true;
      if (s.num_int && (c == '.' || c == 'e' || c == 'E')) return false;
      if (c == '.') { s.lex = L_NUM_DOT; return true; }
      if (c == 'e' || c == 'E') { s.lex = L_NUM_E; return true; }
      return s_end_number(sc, s, c);
    case L_NUM_FRAC:
      if (is_digit(c)) return true;
      if (c == 'e' || c == 'E') { s.lex = L_NUM_E; return true; }
      return s_end_number(sc, s, c);
    case L_NUM_EXP:
      if (is_digit(c)) return true;
      return s_end_number(sc, s, c);
    case L_LIT:
      if (c != (uint8_t)kLits[s.lit][s.lit_pos]) return false;
      if (++s.lit_pos == kLitLen[s.lit]) s_value_done(s);
      return true;
    default: {
      // escapes, \u digits and the number states that cannot end a value: the generic rules
      State g;
      g.lex = s.lex;
      if (!step(g, c)) return false;
      s.lex = g.lex;
      return true;
    }
  }
}

inline bool s_complete(const SState& s) { return s.depth == 0 && s.done && s.lex == L_STRUCT; }

}  // namespace

class SchemaMatcher {
 public:
  SchemaMatcher(std::shared_ptr<VocabIndex> vi, std::shared_ptr<Schema> sc, int64_t max_ws)
      : vi_(std::move(vi)), sc_(std::move(sc)) {
    s_.max_ws = (uint8_t)std::min<int64_t>(std::max<int64_t>(max_ws, 1), 255);
  }
  bool advance(int64_t tok) {
    if (tok == vi_->eos()) {
      if (!s_complete(s_)) return false;
      terminated_ = true;
      return true;
    }
    if (tok < 0 || tok >= (int64_t)vi_->vocab() || vi_->bytes_of(tok).empty()) return false;
    SState t = s_;
    for (unsigned char c : vi_->bytes_of(tok))
      if (!s_step(*sc_, t, c)) return false;
    s_ = t;
    return true;
  }
  bool is_complete() const { return s_complete(s_); }
  bool is_terminated() const { return terminated_ || s_complete(s_); }
  torch::Tensor allowed_mask() const {
    const int words = (vi_->vocab() + 31) / 32;
    auto out = torch::zeros({words}, torch::kInt32);
    uint32_t* m = reinterpret_cast<uint32_t*>(out.data_ptr<int32_t>());
    if (s_.lex == L_STR) {  // free string content: the plain-string tokens, then the others
      std::memcpy(m, vi_->plain().data(), sizeof(uint32_t) * words);
      walk(vi_->special(), 0, s_, m);
    } else {
      walk(vi_->full(), 0, s_, m);
    }
    const int e = vi_->eos();
    if (s_complete(s_) && e >= 0 && e < vi_->vocab()) m[e >> 5] |= 1u << (e & 31);
    return out;
  }

 private:
  void walk(const std::vector<VocabIndex::Node>& t, int n, const SState& s, uint32_t* m) const {
    for (int id : t[n].ends) m[id >> 5] |= 1u << (id & 31);
    for (const auto& kc : t[n].kids) {
      SState c = s;
      if (s_step(*sc_, c, kc.first)) walk(t, kc.second, c, m);
    }
  }
  std::shared_ptr<VocabIndex> vi_;
  std::shared_ptr<Schema> sc_;
  SState s_;
  bool terminated_ = false;
};

void register_grammar(pybind11::module& m) {
  auto g = m.def_submodule("grammar", "JSON-constrained decoding: token bitmasks");
  pybind11::class_<VocabIndex, std::shared_ptr<VocabIndex>>(g, "VocabIndex")
      .def(pybind11::init([](const std::vector<pybind11::bytes>& toks, int64_t eos) {
        std::vector<std::string> v;
        v.reserve(toks.size());
        for (const auto& b : toks) v.push_back(std::string(b));
        return std::make_shared<VocabIndex>(std::move(v), eos);
      }))
      .def_property_readonly("vocab", &VocabIndex::vocab)
      .def("nodes", [](const VocabIndex& v) { return std::make_pair(v.full().size(), v.special().size()); });
  pybind11::class_<JsonMatcher>(g, "JsonMatcher")
      .def(pybind11::init<std::shared_ptr<VocabIndex>, bool, int64_t>(), pybind11::arg("index"),
           pybind11::arg("top_object") = true, pybind11::arg("max_ws") = 24)
      .def("advance", &JsonMatcher::advance)
      .def("allowed_mask", &JsonMatcher::allowed_mask)
      .def("is_complete", &JsonMatcher::is_complete)
      .def("is_terminated", &JsonMatcher::is_terminated);
  pybind11::class_<Schema, std::shared_ptr<Schema>>(g, "Schema")
      .def(pybind11::init<const std::vector<int64_t>&,
                          const std::vector<std::vector<std::pair<pybind11::bytes, int64_t>>>&,
                          const std::vector<int64_t>&, const std::vector<int64_t>&,
                          const std::vector<std::vector<pybind11::bytes>>&, int64_t>());
  pybind11::class_<SchemaMatcher>(g, "SchemaMatcher")
      .def(pybind11::init<std::shared_ptr<VocabIndex>, std::shared_ptr<Schema>, int64_t>(), pybind11::arg("index"),
           pybind11::arg("schema"), pybind11::arg("max_ws") = 24)
      .def("advance", &SchemaMatcher::advance)
      .def("allowed_mask", &SchemaMatcher::allowed_mask)
      .def("is_complete", &SchemaMatcher::is_complete)
      .def("is_terminated", &SchemaMatcher::is_terminated);
}

}  // namespace sqgram

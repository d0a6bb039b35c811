// tokenizer.cpp — the prompt tokenizer of the pi0.5 wrapper: a SentencePiece BPE model read from its
// .model file and the pi0.5 prompt layout (the reference's C++ tokenizer, docs/archive/windows/
// π05_네이티브엔진.md:83 — "SentencePiece BPE, byte fallback, user-defined symbols", checked there against
// Python sentencepiece on 4040 sentences).  Host code.
//
// Model file: a protobuf ModelProto (the SentencePiece model format): field 1 pieces {1 piece, 2 score
// (float), 3 type (1 normal, 2 unknown, 3 control, 4 user-defined, 5 unused, 6 byte)}, field 2 trainer
// spec {3 model_type (2 = BPE), 35 byte_fallback, 40 unk_id, 41 bos_id, 42 eos_id, 43 pad_id}, field 3
// normalizer spec {1 name, 2 precompiled_charsmap, 3 add_dummy_prefix, 4 remove_extra_whitespaces,
// 5 escape_whitespaces}.  Only BPE models with identity normalization (no character map; Gemma's
// tokenizer is one) are accepted.
//
// Encoding (the published SentencePiece BPE algorithm): normalize (drop leading, trailing and repeated
// spaces when remove_extra_whitespaces; prepend a space when add_dummy_prefix; spaces become U+2581
// when escape_whitespaces); split into UTF-8 characters, user-defined symbols matched first (longest)
// and never merged; then repeatedly merge the adjacent pair whose concatenation is a vocabulary piece
// of the highest score (leftmost on ties); unused pieces are split back into the pair that formed them;
// a symbol outside the vocabulary becomes its UTF-8 bytes' <0xXX> pieces with byte fallback, else unk
// (a run of unknown symbols then being one unk).
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/pi05.h"

struct pi05_tokenizer {
  struct Piece {
    std::string s;
    float score = 0.f;
    int type = 1;
  };
  std::vector<Piece> pieces;
  std::unordered_map<std::string, int> normal;    // normal, user-defined and unused pieces (mergeable)
  std::unordered_map<std::string, int> reserved;  // control, unknown and byte pieces
  std::vector<std::string> user_defined;
  int unk_id = 0, bos_id = 1, eos_id = 2, pad_id = -1;
  bool byte_fallback = false;
  bool add_dummy_prefix = true, remove_extra_ws = true, escape_ws = true;
};

namespace {

// ---------------------------------------------------------------- protobuf wire format
struct Pb {
  const uint8_t* p;
  const uint8_t* e;
  bool ok = true;
  uint64_t varint() {
    uint64_t v = 0;
    for (int s = 0; s < 64; s += 7) {
      if (p >= e) {
        ok = false;
        return 0;
      }
      const uint8_t b = *p++;
      v |= (uint64_t)(b & 0x7f) << s;
      if (!(b & 0x80)) return v;
    }
    ok = false;
    return v;
  }
  // next field: number, wire type; the payload is consumed by the caller through the helpers below
  bool next(int* field, int* wt) {
    if (p >= e || !ok) return false;
    const uint64_t k = varint();
    *field = (int)(k >> 3);
    *wt = (int)(k & 7);
    return ok;
  }
  std::string bytes() {
    const uint64_t n = varint();
    if (!ok || n > (uint64_t)(e - p)) {
      ok = false;
      return {};
    }
    std::string s((const char*)p, (size_t)n);
    p += n;
    return s;
  }
  float f32() {
    if (e - p < 4) {
      ok = false;
      return 0.f;
    }
    float f;
    memcpy(&f, p, 4);
    p += 4;
    return f;
  }
  void skip(int wt) {
    if (wt == 0) varint();
    else if (wt == 1) p = (e - p >= 8) ? p + 8 : (ok = false, e);
    else if (wt == 2) bytes();
    else if (wt == 5) p = (e - p >= 4) ? p + 4 : (ok = false, e);
    else ok = false;
  }
};

bool parse_model(const std::string& buf, pi05_tokenizer* t, std::string& err) {
  Pb pb{(const uint8_t*)buf.data(), (const uint8_t*)buf.data() + buf.size()};
  int f, wt, model_type = 1;
  std::string charsmap;
  while (pb.next(&f, &wt)) {
    if (f == 1 && wt == 2) {
      const std::string m = pb.bytes();
      Pb q{(const uint8_t*)m.data(), (const uint8_t*)m.data() + m.size()};
      pi05_tokenizer::Piece pc;
      int g, w2;
      while (q.next(&g, &w2)) {
        if (g == 1 && w2 == 2) pc.s = q.bytes();
        else if (g == 2 && w2 == 5) pc.score = q.f32();
        else if (g == 3 && w2 == 0) pc.type = (int)q.varint();
        else q.skip(w2);
      }
      if (!q.ok) break;
      t->pieces.push_back(pc);
    } else if ((f == 2 || f == 3) && wt == 2) {
      const std::string m = pb.bytes();
      Pb q{(const uint8_t*)m.data(), (const uint8_t*)m.data() + m.size()};
      int g, w2;
      while (q.next(&g, &w2)) {
        if (f == 2 && w2 == 0 && (g == 3 || g == 35 || (g >= 40 && g <= 43))) {
          const int64_t v = (int64_t)q.varint();
          if (g == 3) model_type = (int)v;
          if (g == 35) t->byte_fallback = v != 0;
          if (g == 40) t->unk_id = (int)v;
          if (g == 41) t->bos_id = (int)(int32_t)v;
          if (g == 42) t->eos_id = (int)(int32_t)v;
          if (g == 43) t->pad_id = (int)(int32_t)v;
        } else if (f == 3 && g == 2 && w2 == 2) {
          charsmap = q.bytes();
        } else if (f == 3 && w2 == 0 && g >= 3 && g <= 5) {
          const bool v = q.varint() != 0;
          if (g == 3) t->add_dummy_prefix = v;
          if (g == 4) t->remove_extra_ws = v;
          if (g == 5) t->escape_ws = v;
        } else {
          q.skip(w2);
        }
      }
      if (!q.ok) pb.ok = false;
    } else {
      pb.skip(wt);
    }
  }
  if (!pb.ok || t->pieces.empty()) {
    err = "not a SentencePiece model file";
    return false;
  }
  if (model_type != 2) {
    err = "only BPE SentencePiece models are supported";
    return false;
  }
  if (!charsmap.empty()) {
    err = "only identity normalization is supported (the model has a character map)";
    return false;
  }
  for (int i = 0; i < (int)t->pieces.size(); ++i) {
    const auto& pc = t->pieces[i];
    const bool mergeable = pc.type == 1 || pc.type == 4 || pc.type == 5;
    auto& m = mergeable ? t->normal : t->reserved;
    if (!m.emplace(pc.s, i).second) {
      err = "duplicate piece " + pc.s;
      return false;
    }
    if (pc.type == 4) t->user_defined.push_back(pc.s);
    if (pc.type == 2) t->unk_id = i;
  }
  return true;
}

int char_len(uint8_t c) {
  static const int tab[16] = {1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 2, 2, 3, 4};
  return tab[c >> 4];
}

std::string normalize(const pi05_tokenizer* t, const std::string& in) {
  std::string s;
  size_t i = 0;
  if (t->remove_extra_ws)
    while (i < in.size() && in[i] == ' ') ++i;
  bool prev_space = false;
  for (; i < in.size(); ++i) {
    const char c = in[i];
    if (c == ' ') {
      if (t->remove_extra_ws && prev_space) continue;
      prev_space = true;
    } else {
      prev_space = false;
    }
    s.push_back(c);
  }
  if (t->remove_extra_ws)
    while (!s.empty() && s.back() == ' ') s.pop_back();
  if (t->add_dummy_prefix && !s.empty()) s.insert(0, " ");
  if (!t->escape_ws) return s;
  std::string o;
  for (char c : s) o += c == ' ' ? std::string("\xe2\x96\x81") : std::string(1, c);
  return o;
}

struct Sym {
  std::string piece;
  int prev, next;
  bool freeze;
};

struct Pair {
  int left, right;
  float score;
  size_t size;
};

struct PairOrder {
  bool operator()(const Pair& a, const Pair& b) const {
    return a.score < b.score || (a.score == b.score && a.left > b.left);
  }
};

void resegment(const pi05_tokenizer* t, const std::string& w,
               const std::unordered_map<std::string, std::pair<std::string, std::string>>& rev,
               std::vector<int>& out) {
  auto it = t->normal.find(w);
  if (it != t->normal.end() && t->pieces[it->second].type == 5) {
    auto r = rev.find(w);
    if (r != rev.end()) {
      resegment(t, r->second.first, rev, out);
      resegment(t, r->second.second, rev, out);
      return;
    }
  }
  if (it != t->normal.end()) {
    out.push_back(it->second);
    return;
  }
  auto rs = t->reserved.find(w);
  if (rs != t->reserved.end() && t->pieces[rs->second].type != 6) {  // control / unknown spelled out
    out.push_back(rs->second);
    return;
  }
  if (t->byte_fallback) {
    for (unsigned char b : w) {
      char name[8];
      snprintf(name, sizeof name, "<0x%02X>", b);
      auto bt = t->reserved.find(name);
      out.push_back(bt != t->reserved.end() ? bt->second : t->unk_id);
    }
    return;
  }
  out.push_back(t->unk_id);
}

std::vector<int> encode(const pi05_tokenizer* t, const std::string& text) {
  const std::string norm = normalize(t, text);
  std::vector<Sym> sy;
  for (size_t i = 0; i < norm.size();) {
    size_t len = 0;
    for (const std::string& u : t->user_defined)
      if (u.size() > len && norm.compare(i, u.size(), u) == 0) len = u.size();
    const bool freeze = len > 0;
    if (!freeze) len = std::min((size_t)char_len((uint8_t)norm[i]), norm.size() - i);
    const int idx = (int)sy.size();
    sy.push_back({norm.substr(i, len), idx - 1, -1, freeze});
    if (idx > 0) sy[idx - 1].next = idx;
    i += len;
  }
  std::priority_queue<Pair, std::vector<Pair>, PairOrder> agenda;
  std::unordered_map<std::string, std::pair<std::string, std::string>> rev;
  auto add = [&](int l, int r) {
    if (l < 0 || r < 0 || sy[l].freeze || sy[r].freeze) return;
    const std::string m = sy[l].piece + sy[r].piece;
    auto it = t->normal.find(m);
    if (it == t->normal.end()) return;
    agenda.push({l, r, t->pieces[it->second].score, m.size()});
    if (t->pieces[it->second].type == 5) rev[m] = {sy[l].piece, sy[r].piece};
  };
  for (int i = 1; i < (int)sy.size(); ++i) add(i - 1, i);
  while (!agenda.empty()) {
    const Pair p = agenda.top();
    agenda.pop();
    if (sy[p.left].piece.empty() || sy[p.right].piece.empty() ||
        sy[p.left].piece.size() + sy[p.right].piece.size() != p.size)
      continue;  // a neighbour merged since this pair was queued
    sy[p.left].piece += sy[p.right].piece;
    sy[p.right].piece.clear();
    sy[p.left].next = sy[p.right].next;
    if (sy[p.right].next >= 0) sy[sy[p.right].next].prev = p.left;
    add(sy[p.left].prev, p.left);
    add(p.left, sy[p.left].next);
  }
  std::vector<int> out;
  for (int i = sy.empty() ? -1 : 0; i >= 0; i = sy[i].next) resegment(t, sy[i].piece, rev, out);
  if (!t->byte_fallback) {  // a run of unknown symbols is one unknown piece
    std::vector<int> merged;
    for (int id : out)
      if (!(id == t->unk_id && !merged.empty() && merged.back() == t->unk_id)) merged.push_back(id);
    out.swap(merged);
  }
  return out;
}

}  // namespace

extern "C" {

pi05_tokenizer* pi05_tokenizer_load(const char* path, char* err, size_t err_len) {
  auto fail = [&](const std::string& m) -> pi05_tokenizer* {
    if (err && err_len) snprintf(err, err_len, "%s", m.c_str());
    return nullptr;
  };
  if (!path) return fail("pi05_tokenizer_load: no path");
  FILE* f = fopen(path, "rb");
  if (!f) return fail(std::string("pi05_tokenizer_load: cannot open ") + path);
  std::string buf;
  char chunk[65536];
  size_t n;
  while ((n = fread(chunk, 1, sizeof chunk, f)) > 0) buf.append(chunk, n);
  fclose(f);
  pi05_tokenizer* t = new pi05_tokenizer();
  std::string e;
  if (!parse_model(buf, t, e)) {
    delete t;
    return fail("pi05_tokenizer_load: " + e);
  }
  return t;
}

void pi05_tokenizer_free(pi05_tokenizer* t) { delete t; }

int pi05_tokenizer_vocab_size(const pi05_tokenizer* t) { return t ? (int)t->pieces.size() : 0; }

int pi05_tokenizer_encode(const pi05_tokenizer* t, const char* text, int add_bos, int32_t* ids, int max_ids) {
  if (!t || !text || (max_ids > 0 && !ids) || max_ids < 0) return PI05_ERR_ARG;
  std::vector<int> v = encode(t, text);
  if (add_bos && t->bos_id >= 0) v.insert(v.begin(), t->bos_id);
  for (int i = 0; i < (int)v.size() && i < max_ids; ++i) ids[i] = v[i];
  return (int)v.size();
}

int pi05_tokenize_prompt(const pi05_tokenizer* t, const char* task, const float* state, int state_dim, int max_len,
                         int32_t* ids, uint8_t* mask) {
  if (!t || !task || max_len < 1 || !ids || state_dim < 0 || (state_dim > 0 && !state)) return PI05_ERR_ARG;
  // openpi's prompt cleaning: strip surrounding whitespace, '_' and '\n' become spaces
  std::string s = task;
  const char* ws = " \t\n\r\f\v";
  const size_t a = s.find_first_not_of(ws), b = s.find_last_not_of(ws);
  s = a == std::string::npos ? std::string() : s.substr(a, b - a + 1);
  for (char& c : s)
    if (c == '_' || c == '\n') c = ' ';
  std::string full;
  if (state_dim > 0) {
    std::vector<int32_t> bins(state_dim);
    pi05_discretize_state(state, 1, state_dim, 256, bins.data());
    std::string st;
    for (int i = 0; i < state_dim; ++i) st += (i ? " " : "") + std::to_string(bins[i]);
    full = "Task: " + s + ", State: " + st + ";\nAction: ";
  } else {
    full = s;
  }
  std::vector<int> v = encode(t, full);
  if (t->bos_id >= 0) v.insert(v.begin(), t->bos_id);
  if (state_dim == 0) {  // the pi0 layout: "\n" encoded on its own closes the prompt
    const std::vector<int> nl = encode(t, "\n");
    v.insert(v.end(), nl.begin(), nl.end());
  }
  const int n = (int)std::min<size_t>(v.size(), (size_t)max_len);
  for (int i = 0; i < max_len; ++i) {
    ids[i] = i < n ? v[i] : 0;
    if (mask) mask[i] = i < n;
  }
  return n;
}

}  // extern "C"

// Streaming text of many sessions decoded together: the host path that turns
// each step's next tokens into text while the GPU runs the next step.
//
// Per session it restates the reference's two streaming stages:
//  * Utf8Stream (tokenizer/src/stream.rs:48-131): token pieces are raw bytes
//    that may end inside a UTF-8 sequence; the completed prefix is emitted,
//    an incomplete tail is kept, and a sequence that can never become valid is
//    either an error (the buffer is kept) or one U+FFFD per maximal invalid
//    subsequence (the String::from_utf8_lossy rule);
//  * DecodedText (engine/src/text_output.rs:9-53): the whole-sequence
//    clean_spaces pass of the tokenizer's decoder recomputed over the text so
//    far, with the last 16 bytes withheld until the next chunk (or the end).
// Token pieces come from the caller (the tokenizer's token_to_piece for every
// id, which owns the vocabulary rules); this file only assembles them.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/lfm_cuda.h"

namespace {

thread_local std::string t_text_err;

// Length of the longest valid UTF-8 prefix of p[0, n), and for the first
// problem after it: *bad = bytes of a maximal invalid subsequence (1..3) or 0
// when the rest is an incomplete (still completable) sequence at the end.
// Well-formed sequences per the Unicode table (no overlongs, no surrogates,
// nothing above U+10FFFF), the rule of Rust's str::from_utf8.
size_t utf8_valid_prefix(const uint8_t* p, size_t n, size_t* bad) {
  size_t i = 0;
  *bad = 0;
  while (i < n) {
    const uint8_t c = p[i];
    if (c < 0x80) {
      i++;
      continue;
    }
    int len;
    uint8_t lo = 0x80, hi = 0xBF;  // range of the second byte
    if (c >= 0xC2 && c <= 0xDF) len = 2;
    else if (c == 0xE0) len = 3, lo = 0xA0;
    else if (c >= 0xE1 && c <= 0xEC) len = 3;
    else if (c == 0xED) len = 3, hi = 0x9F;
    else if (c >= 0xEE && c <= 0xEF) len = 3;
    else if (c == 0xF0) len = 4, lo = 0x90;
    else if (c >= 0xF1 && c <= 0xF3) len = 4;
    else if (c == 0xF4) len = 4, hi = 0x8F;
    else {
      *bad = 1;
      return i;
    }
    for (int k = 1; k < len; k++) {
      if (i + k >= n) return i;  // incomplete at the end: *bad stays 0
      const uint8_t b = p[i + k];
      const bool ok = k == 1 ? (b >= lo && b <= hi) : (b >= 0x80 && b <= 0xBF);
      if (!ok) {
        *bad = (size_t)k;
        return i;
      }
    }
    i += (size_t)len;
  }
  return i;
}

// vocab.rs clean_spaces / text_output.rs:59-106 (llama.cpp's detokenizer
// passes: " ?" " !" " ." " ," lose the space; " ' " between spaces; " 's",
// " 'm", " 're", " 've" lose the space), same in-place index arithmetic.
void clean_spaces(std::string& text) {
  size_t total = text.size();
  const size_t total1 = total;
  total = total > 0 ? 1 : 0;
  for (size_t i = 1; i < total1; i++) {
    const char x = text[i];
    if (text[i - 1] == ' ' && (x == '?' || x == '!' || x == '.' || x == ',')) total--;
    text[total++] = x;
  }
  const size_t total2 = total;
  total = total > 0 ? 1 : 0;
  size_t i = 1;
  while (i < total2) {
    const char x = text[i];
    if (x == '\'' && i + 1 < total2 && text[i - 1] == ' ' && text[i + 1] == ' ') {
      total--;
      i++;
      text[i] = 0;
    }
    text[total++] = x;
    i++;
  }
  const size_t total3 = total;
  total = total > 0 ? 1 : 0;
  for (size_t j = 1; j < total3; j++) {
    const char x = text[j];
    if (text[j - 1] == ' ' && x == '\'' && j + 1 < total3) {
      const char x1 = text[j + 1];
      if (x1 == 't' || x1 == 'd') {
      } else if (x1 == 's' || x1 == 'm') {
        total--;
      } else if (j + 2 < total3) {
        const char x2 = text[j + 2];
        if (x1 == 'l' && x2 == 'l') {
        } else if ((x1 == 'r' && x2 == 'e') || (x1 == 'v' && x2 == 'e')) {
          total--;
        }
      }
    }
    text[total++] = x;
  }
  text.resize(total);
}

bool is_char_boundary(const std::string& s, size_t i) {
  return i == 0 || i >= s.size() || ((uint8_t)s[i] & 0xC0) != 0x80;
}

struct Session {
  std::string pending;   // Utf8Stream: bytes of an incomplete trailing sequence
  std::string raw;       // DecodedText: every completed chunk so far
  std::string emitted;   // DecodedText: the text returned so far
  uint64_t tokens = 0;
};

}  // namespace

struct lfm_text {
  std::vector<uint64_t> off;   // piece of token t: bytes[off[t], off[t + 1])
  std::string bytes;
  bool clean = true, replace = false;
  std::vector<Session> sess;

  // Utf8Stream::push: append, return the completed text (false: invalid bytes
  // under the error policy; the buffer keeps them).
  bool utf8_push(Session& s, const char* p, size_t n, std::string& out) {
    s.pending.append(p, n);
    size_t consumed = 0;
    for (;;) {
      const uint8_t* rest = (const uint8_t*)s.pending.data() + consumed;
      const size_t left = s.pending.size() - consumed;
      size_t bad;
      const size_t good = utf8_valid_prefix(rest, left, &bad);
      out.append((const char*)rest, good);
      if (good == left) {
        consumed = s.pending.size();
        break;
      }
      if (bad == 0) {  // incomplete sequence at the end: keep it
        consumed += good;
        break;
      }
      if (!replace) {
        t_text_err = "invalid UTF-8 (valid up to byte " + std::to_string(consumed + good) + " of the buffered piece bytes)";
        return false;
      }
      out.append("\xEF\xBF\xBD");
      consumed += good + bad;
    }
    s.pending.erase(0, consumed);
    return true;
  }

  // DecodedText::push / finish; false if the cleanup changed text that was
  // already emitted (the reference asserts that it cannot).
  bool take(Session& s, const std::string& chunk, bool final_chunk, std::string& delta) {
    s.raw += chunk;
    std::string text = s.raw;
    if (clean) clean_spaces(text);
    size_t end = (final_chunk || !clean) ? text.size() : (text.size() > 16 ? text.size() - 16 : 0);
    while (!is_char_boundary(text, end)) end--;
    if (text.compare(0, s.emitted.size(), s.emitted) != 0) {
      t_text_err = "cleanup changed an already-emitted prefix";
      return false;
    }
    end = std::max(end, s.emitted.size());
    delta = text.substr(s.emitted.size(), end - s.emitted.size());
    s.emitted += delta;
    return true;
  }
};

extern "C" {

lfm_status lfm_text_create(const uint8_t* piece_bytes, const uint64_t* piece_off, uint32_t n_tokens,
                           uint32_t n_sessions, int clean_spaces_on, int replace_invalid, lfm_text** out) {
  if (!out || !piece_off || n_tokens == 0 || n_sessions == 0 || (!piece_bytes && piece_off[n_tokens] > 0)) {
    t_text_err = "lfm_text_create: bad argument";
    return LFM_ERR_ARG;
  }
  for (uint32_t t = 0; t < n_tokens; t++)
    if (piece_off[t + 1] < piece_off[t]) {
      t_text_err = "lfm_text_create: piece offsets must not decrease";
      return LFM_ERR_ARG;
    }
  auto* T = new lfm_text();
  T->off.assign(piece_off, piece_off + n_tokens + 1);
  T->bytes.assign((const char*)piece_bytes + piece_off[0], (size_t)(piece_off[n_tokens] - piece_off[0]));
  for (auto& o : T->off) o -= piece_off[0];
  T->clean = clean_spaces_on != 0;
  T->replace = replace_invalid != 0;
  T->sess.resize(n_sessions);
  *out = T;
  return LFM_OK;
}

void lfm_text_destroy(lfm_text* t) { delete t; }

lfm_status lfm_text_push(lfm_text* t, const uint32_t* sessions, const uint32_t* tokens, uint32_t count, char* out,
                         size_t cap, uint64_t* out_off) {
  if (!t || (count && (!sessions || !tokens || !out_off)) || (!out && cap)) {
    t_text_err = "lfm_text_push: bad argument";
    return LFM_ERR_ARG;
  }
  const uint32_t ntok = (uint32_t)t->off.size() - 1;
  for (uint32_t i = 0; i < count; i++)
    if (sessions[i] >= t->sess.size() || tokens[i] >= ntok) {
      t_text_err = "lfm_text_push: session or token id out of range (entry " + std::to_string(i) + ")";
      return LFM_ERR_ARG;
    }
  size_t w = 0;
  out_off[0] = 0;
  std::string chunk, delta;
  for (uint32_t i = 0; i < count; i++) {
    Session& s = t->sess[sessions[i]];
    const uint32_t id = tokens[i];
    chunk.clear();
    if (!t->utf8_push(s, t->bytes.data() + t->off[id], (size_t)(t->off[id + 1] - t->off[id]), chunk)) {
      t_text_err = "session " + std::to_string(sessions[i]) + ": " + t_text_err;
      return LFM_ERR_STATE;
    }
    s.tokens++;
    if (!t->take(s, chunk, false, delta)) return LFM_ERR_STATE;
    if (w + delta.size() > cap) {
      t_text_err = "lfm_text_push: output buffer too small";
      return LFM_ERR_ARG;
    }
    memcpy(out + w, delta.data(), delta.size());
    w += delta.size();
    out_off[i + 1] = w;
  }
  return LFM_OK;
}

lfm_status lfm_text_finish(lfm_text* t, uint32_t session, char* out, size_t cap, size_t* len) {
  if (!t || session >= t->sess.size() || !len || (!out && cap)) {
    t_text_err = "lfm_text_finish: bad argument";
    return LFM_ERR_ARG;
  }
  Session& s = t->sess[session];
  std::string tail;
  lfm_status st = LFM_OK;
  if (!s.pending.empty()) {
    // Utf8Stream::finish: an incomplete tail is an error, or one U+FFFD
    size_t bad;
    const size_t good = utf8_valid_prefix((const uint8_t*)s.pending.data(), s.pending.size(), &bad);
    if (t->replace) {
      tail = "\xEF\xBF\xBD";
    } else if (good == s.pending.size()) {
      tail = s.pending;
    } else {
      t_text_err = bad ? "invalid UTF-8 at the end of the stream" : "incomplete UTF-8 sequence at the end of the stream";
      st = LFM_ERR_STATE;
    }
  }
  std::string delta;
  if (st == LFM_OK && !t->take(s, tail, true, delta)) st = LFM_ERR_STATE;
  s = Session();  // finish leaves the session empty, ready for a new stream
  if (delta.size() > cap) {
    t_text_err = "lfm_text_finish: output buffer too small";
    return LFM_ERR_ARG;
  }
  if (!delta.empty()) memcpy(out, delta.data(), delta.size());
  *len = delta.size();
  return st;
}

lfm_status lfm_text_reset(lfm_text* t, uint32_t session) {
  if (!t || session >= t->sess.size()) {
    t_text_err = "lfm_text_reset: bad argument";
    return LFM_ERR_ARG;
  }
  t->sess[session] = Session();
  return LFM_OK;
}

const char* lfm_text_error(void) { return t_text_err.c_str(); }

}  // extern "C"

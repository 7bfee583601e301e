// Host tokenizer: a C++ restatement of internal/embed/tokenizer.go behind the
// C ABI (include/llmembed.h le_tokenizer_*), multithreaded over texts.
//
// Encode (tokenizer.go:47-80): Go's strings.ToLower (unicode.ToLower per
// rune; invalid UTF-8 bytes become U+FFFD), split into words on Go's
// unicode.IsSpace and BERT punctuation (ASCII punctuation, general category
// P*, the CJK ideograph blocks; each punctuation rune is a word of its own),
// greedy longest match per word over its UTF-8 bytes with the U+2581 prefix
// on the first piece (pieces at most the longest vocabulary entry), then a
// single byte with the prefix (first piece only), a single byte, or
// [UNK]=100 per byte (encodeWord, tokenizer.go:84-142); [CLS]=101 ...
// [SEP]=102, truncated to max_len with [SEP] kept last.  The vocabulary is
// token -> id with later duplicates winning, as a Go map assignment does
// (LoadTokenizer, tokenizer.go:24-44).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstring>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "../../include/llmembed.h"
#include "unicode_tables.h"

int le_fail(int code, const char* fmt, ...);  // api.cu: sets le_last_error

namespace {

constexpr int CLS = 101, SEP = 102, UNK = 100;
const char PREFIX[3] = {'\xE2', '\x96', '\x81'};  // U+2581

// ------------------------------------------------------------ Unicode --

uint32_t to_lower(uint32_t r) {
  if (r < 0x80) return (r >= 'A' && r <= 'Z') ? r + 32 : r;
  int lo = 0, hi = le::uni::N_LOWER - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const uint32_t c = le::uni::LOWER[mid][0];
    if (c == r) return le::uni::LOWER[mid][1];
    if (c < r) lo = mid + 1;
    else hi = mid - 1;
  }
  return r;
}

bool is_space(uint32_t r) {
  if (r < 0x100) return r == '\t' || r == '\n' || r == '\v' || r == '\f' || r == '\r' || r == ' ' || r == 0x85 ||
                        r == 0xA0;
  for (int i = 0; i < le::uni::N_SPACE_HI; i++)
    if (le::uni::SPACE_HI[i] == r) return true;
  return false;
}

bool is_bert_punct(uint32_t r) {
  if ((r >= '!' && r <= '/') || (r >= ':' && r <= '@') || (r >= '[' && r <= '`') || (r >= '{' && r <= '~'))
    return true;
  if ((r >= 0x4E00 && r <= 0x9FFF) || (r >= 0x3400 && r <= 0x4DBF) || (r >= 0x20000 && r <= 0x2A6DF)) return true;
  if (r < 0x80) return false;
  int lo = 0, hi = le::uni::N_PUNCT - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (r < le::uni::PUNCT[mid][0]) hi = mid - 1;
    else if (r > le::uni::PUNCT[mid][1]) lo = mid + 1;
    else return true;
  }
  return false;
}

// One rune of UTF-8 at p (n bytes left) as Go's range loop decodes it:
// invalid or truncated sequences, surrogates and overlong forms give
// U+FFFD and advance one byte.
uint32_t decode(const uint8_t* p, size_t n, int* len) {
  const uint8_t b0 = p[0];
  *len = 1;
  if (b0 < 0x80) return b0;
  auto cont = [&](size_t i) { return i < n && (p[i] & 0xC0) == 0x80; };
  if (b0 >= 0xC2 && b0 <= 0xDF && cont(1)) {
    *len = 2;
    return ((b0 & 0x1Fu) << 6) | (p[1] & 0x3Fu);
  }
  if (b0 >= 0xE0 && b0 <= 0xEF && cont(1) && cont(2)) {
    const uint32_t r = ((b0 & 0x0Fu) << 12) | ((p[1] & 0x3Fu) << 6) | (p[2] & 0x3Fu);
    if (r >= 0x800 && (r < 0xD800 || r > 0xDFFF)) {
      *len = 3;
      return r;
    }
    return 0xFFFD;
  }
  if (b0 >= 0xF0 && b0 <= 0xF4 && cont(1) && cont(2) && cont(3)) {
    const uint32_t r = ((b0 & 0x07u) << 18) | ((p[1] & 0x3Fu) << 12) | ((p[2] & 0x3Fu) << 6) | (p[3] & 0x3Fu);
    if (r >= 0x10000 && r <= 0x10FFFF) {
      *len = 4;
      return r;
    }
  }
  return 0xFFFD;
}

void encode_utf8(uint32_t r, std::string& out) {
  if (r < 0x80) {
    out.push_back((char)r);
  } else if (r < 0x800) {
    out.push_back((char)(0xC0 | (r >> 6)));
    out.push_back((char)(0x80 | (r & 0x3F)));
  } else if (r < 0x10000) {
    out.push_back((char)(0xE0 | (r >> 12)));
    out.push_back((char)(0x80 | ((r >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (r & 0x3F)));
  } else {
    out.push_back((char)(0xF0 | (r >> 18)));
    out.push_back((char)(0x80 | ((r >> 12) & 0x3F)));
    out.push_back((char)(0x80 | ((r >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (r & 0x3F)));
  }
}

// ------------------------------------------------------------ vocabulary --

uint64_t hash_bytes(const char* p, size_t n) {
  uint64_t h = 1469598103934665603ull;  // FNV-1a, then a final mix
  for (size_t i = 0; i < n; i++) h = (h ^ (uint8_t)p[i]) * 1099511628211ull;
  h ^= h >> 29;
  h *= 0xBF58476D1CE4E5B9ull;
  return h ^ (h >> 32);
}

}  // namespace

struct le_tokenizer {
  std::string bytes;            // all tokens back to back
  std::vector<uint64_t> off;    // token i = bytes[off[i], off[i+1])
  std::vector<int32_t> slots;   // open addressing: token id or -1
  uint64_t mask = 0;
  size_t max_token = 0;

  bool eq(int32_t id, const char* p, size_t n) const {
    return off[id + 1] - off[id] == n && std::memcmp(bytes.data() + off[id], p, n) == 0;
  }
  // id of the token with these bytes, or -1.
  int32_t find(const char* p, size_t n) const {
    for (uint64_t h = hash_bytes(p, n) & mask;; h = (h + 1) & mask) {
      const int32_t id = slots[h];
      if (id < 0) return -1;
      if (eq(id, p, n)) return id;
    }
  }
  void build(int n) {
    size_t cap = 16;
    while (cap < (size_t)n * 2) cap <<= 1;
    slots.assign(cap, -1);
    mask = cap - 1;
    for (int i = 0; i < n; i++) {
      const char* p = bytes.data() + off[i];
      const size_t len = off[i + 1] - off[i];
      max_token = std::max(max_token, len);
      for (uint64_t h = hash_bytes(p, len) & mask;; h = (h + 1) & mask) {
        if (slots[h] < 0 || eq(slots[h], p, len)) {
          slots[h] = i;  // a later duplicate replaces the earlier id
          break;
        }
      }
    }
  }

  // encodeWord: word = the word's bytes; buf has room for 3 + word bytes.
  void encode_word(const char* w, size_t n, std::string& buf, std::vector<int32_t>& ids) const {
    buf.assign(PREFIX, 3);
    buf.append(w, n);
    int32_t id = find(buf.data(), buf.size());
    if (id >= 0) {
      ids.push_back(id);
      return;
    }
    size_t start = 0;
    while (start < n) {
      size_t end = std::min(n, start + max_token);
      bool found = false;
      while (end > start) {
        // Candidate: prefix + word[0:end] (start == 0) or word[start:end].
        id = start == 0 ? find(buf.data(), 3 + end) : find(w + start, end - start);
        if (id >= 0) {
          ids.push_back(id);
          start = end;
          found = true;
          break;
        }
        end--;
      }
      if (found) continue;
      if (start == 0) {
        id = find(buf.data(), 4);
        if (id >= 0) {
          ids.push_back(id);
          start++;
          continue;
        }
      }
      id = find(w + start, 1);
      ids.push_back(id >= 0 ? id : UNK);
      start++;
    }
  }

  // Encode (tokenizer.go:47-80) of prefix + text into ids (appended).
  void encode(const char* prefix, size_t np, const char* text, size_t nt, int max_len, std::string& lower,
              std::string& buf, std::vector<int32_t>& ids) const {
    const size_t first = ids.size();
    ids.push_back(CLS);
    // strings.ToLower over prefix + text, then preTokenize.
    lower.clear();
    for (int part = 0; part < 2; part++) {
      const uint8_t* p = reinterpret_cast<const uint8_t*>(part ? text : prefix);
      const size_t n = part ? nt : np;
      for (size_t i = 0; i < n;) {
        if (p[i] < 0x80) {
          const uint8_t c = p[i++];
          lower.push_back((char)((c >= 'A' && c <= 'Z') ? c + 32 : c));
          continue;
        }
        int len;
        const uint32_t r = decode(p + i, n - i, &len);
        i += len;
        encode_utf8(to_lower(r), lower);
      }
    }
    const uint8_t* s = reinterpret_cast<const uint8_t*>(lower.data());
    const size_t n = lower.size();
    size_t w0 = 0, i = 0;
    bool in_word = false;
    while (i < n) {
      int len;
      const uint32_t r = decode(s + i, n - i, &len);
      if (is_space(r)) {
        if (in_word) encode_word(lower.data() + w0, i - w0, buf, ids);
        in_word = false;
      } else if (is_bert_punct(r)) {
        if (in_word) encode_word(lower.data() + w0, i - w0, buf, ids);
        in_word = false;
        encode_word(lower.data() + i, (size_t)len, buf, ids);
      } else if (!in_word) {
        in_word = true;
        w0 = i;
      }
      i += len;
    }
    if (in_word) encode_word(lower.data() + w0, n - w0, buf, ids);
    ids.push_back(SEP);
    if (ids.size() - first > (size_t)max_len) {
      ids.resize(first + max_len);
      ids.back() = SEP;
    }
  }
};

namespace {

int make_tokenizer(const std::vector<std::pair<const char*, size_t>>& toks, le_tokenizer** out) {
  auto t = new (std::nothrow) le_tokenizer();
  if (!t) return le_fail(LE_ENOMEM, "tokenizer allocation failed");
  size_t total = 0;
  for (auto& p : toks) total += p.second;
  t->bytes.reserve(total);
  t->off.reserve(toks.size() + 1);
  t->off.push_back(0);
  for (auto& p : toks) {
    t->bytes.append(p.first, p.second);
    t->off.push_back(t->bytes.size());
  }
  t->build((int)toks.size());
  *out = t;
  return LE_OK;
}

}  // namespace

extern "C" {

int le_tokenizer_create(const char* const* tokens, const int32_t* token_lens, int n_tokens, le_tokenizer** out) {
  if (!out || n_tokens < 0 || (n_tokens > 0 && (!tokens || !token_lens))) return le_fail(LE_EINVAL, "null argument");
  *out = nullptr;
  std::vector<std::pair<const char*, size_t>> toks((size_t)n_tokens);
  for (int i = 0; i < n_tokens; i++) {
    if (token_lens[i] < 0 || (token_lens[i] > 0 && !tokens[i])) return le_fail(LE_EINVAL, "bad token %d", i);
    toks[i] = {tokens[i], (size_t)token_lens[i]};
  }
  return make_tokenizer(toks, out);
}

// The string array "tokenizer.ggml.tokens" of a GGUF file's metadata
// (readGGUFStringArray, tokenizer.go:194-250).
int le_tokenizer_load_gguf(const char* path, le_tokenizer** out) {
  if (!path || !out) return le_fail(LE_EINVAL, "null argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return le_fail(LE_EIO, "tokenizer: open %s failed", path);
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    return le_fail(LE_EIO, "tokenizer: stat %s failed", path);
  }
  const size_t n = (size_t)st.st_size;
  void* map = n ? mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  close(fd);
  if (map == MAP_FAILED) return le_fail(LE_EIO, "tokenizer: mmap %s failed", path);
  const uint8_t* p = static_cast<const uint8_t*>(map);
  size_t pos = 0;
  bool ok = true;
  auto need = [&](size_t k) {
    if (pos + k > n) ok = false;
    return ok;
  };
  auto u32 = [&] {
    uint32_t v = 0;
    if (need(4)) std::memcpy(&v, p + pos, 4), pos += 4;
    return v;
  };
  auto u64 = [&] {
    uint64_t v = 0;
    if (need(8)) std::memcpy(&v, p + pos, 8), pos += 8;
    return v;
  };
  std::function<bool(uint32_t)> skip = [&](uint32_t vt) -> bool {
    static const int sizes[13] = {1, 1, 2, 2, 4, 4, 4, 1, -1, -1, 8, 8, 8};
    if (vt > 12) return false;
    if (sizes[vt] > 0) return need(sizes[vt]) && ((pos += sizes[vt]), true);
    if (vt == 8) {
      const uint64_t len = u64();
      return need(len) && ((pos += len), true);
    }
    const uint32_t et = u32();
    const uint64_t cnt = u64();
    for (uint64_t i = 0; i < cnt && ok; i++)
      if (!skip(et)) return false;
    return ok;
  };
  int rc = le_fail(LE_EIO, "tokenizer: key \"tokenizer.ggml.tokens\" not found in %s", path);
  if (need(24) && std::memcmp(p, "GGUF", 4) == 0) {
    pos = 16;
    const uint64_t n_kv = u64();
    static const char KEY[] = "tokenizer.ggml.tokens";
    for (uint64_t k = 0; k < n_kv && ok; k++) {
      const uint64_t klen = u64();
      if (!need(klen)) break;
      const bool match = klen == sizeof(KEY) - 1 && std::memcmp(p + pos, KEY, klen) == 0;
      pos += klen;
      const uint32_t vt = u32();
      if (match && vt == 9) {
        const uint32_t et = u32();
        const uint64_t cnt = u64();
        if (et != 8 || !ok || cnt > (1ull << 31)) {
          rc = le_fail(LE_EIO, "tokenizer: tokenizer.ggml.tokens is not a string array");
          break;
        }
        std::vector<std::pair<const char*, size_t>> toks;
        toks.reserve((size_t)cnt);
        for (uint64_t i = 0; i < cnt && ok; i++) {
          const uint64_t len = u64();
          if (!need(len)) break;
          toks.push_back({reinterpret_cast<const char*>(p + pos), (size_t)len});
          pos += len;
        }
        rc = ok ? make_tokenizer(toks, out) : le_fail(LE_EIO, "tokenizer: truncated GGUF %s", path);
        break;
      }
      if (!skip(vt)) {
        rc = le_fail(LE_EIO, "tokenizer: bad metadata value in %s", path);
        break;
      }
    }
  } else {
    rc = le_fail(LE_EIO, "tokenizer: %s is not a GGUF file", path);
  }
  munmap(map, n);
  return rc;
}

int le_tokenizer_free(le_tokenizer* t) {
  delete t;
  return LE_OK;
}

int le_tokenizer_vocab_size(const le_tokenizer* t, int* n) {
  if (!t || !n) return le_fail(LE_EINVAL, "null argument");
  *n = (int)t->off.size() - 1;
  return LE_OK;
}

int le_tokenize(const le_tokenizer* t, const char* text, const int64_t* text_offsets, int n_texts, const char* prefix,
                int max_len, int32_t* ids, int64_t capacity, int32_t* offsets, int nthreads) {
  if (!t || !offsets || n_texts < 0 || (n_texts > 0 && !text_offsets) || max_len < 2)
    return le_fail(LE_EINVAL, "bad argument");
  for (int i = 0; i < n_texts; i++)
    if (text_offsets[i + 1] < text_offsets[i] || text_offsets[0] < 0)
      return le_fail(LE_EINVAL, "text_offsets not ascending at %d", i);
  if (n_texts > 0 && text_offsets[n_texts] > 0 && !text) return le_fail(LE_EINVAL, "null text");
  const size_t np = prefix ? std::strlen(prefix) : 0;
  if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
  nthreads = std::min(nthreads, std::max(1, n_texts / 16));
  // Texts in chunks of 64, taken dynamically; each chunk's ids kept apart
  // until the offsets are known.
  constexpr int CH = 64;
  const int n_chunks = (n_texts + CH - 1) / CH;
  std::vector<std::vector<int32_t>> chunk_ids((size_t)n_chunks);
  std::vector<std::vector<int32_t>> chunk_len((size_t)n_chunks);
  std::atomic<int> next{0};
  auto work = [&] {
    std::string lower, buf;
    for (int c; (c = next.fetch_add(1)) < n_chunks;) {
      auto& v = chunk_ids[c];
      auto& L = chunk_len[c];
      for (int i = c * CH; i < std::min(n_texts, (c + 1) * CH); i++) {
        const size_t before = v.size();
        const int64_t a = text_offsets[i], b = text_offsets[i + 1];
        t->encode(prefix ? prefix : "", np, b > a ? text + a : "", (size_t)(b - a), max_len, lower, buf, v);
        L.push_back((int32_t)(v.size() - before));
      }
    }
  };
  if (nthreads <= 1) {
    work();
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < nthreads; i++) th.emplace_back(work);
    for (auto& x : th) x.join();
  }
  int64_t total = 0;
  offsets[0] = 0;
  int k = 0;
  for (int c = 0; c < n_chunks; c++)
    for (int32_t len : chunk_len[c]) {
      total += len;
      if (total > INT32_MAX) return le_fail(LE_EINVAL, "more than 2^31 token ids");
      offsets[++k] = (int32_t)total;
    }
  if (total > capacity)
    return le_fail(LE_EINVAL, "ids capacity %lld < %lld token ids (offsets hold the sizes)", (long long)capacity,
                   (long long)total);
  if (total > 0 && !ids) return le_fail(LE_EINVAL, "null ids");
  int64_t at = 0;
  for (int c = 0; c < n_chunks; c++) {
    if (!chunk_ids[c].empty()) std::memcpy(ids + at, chunk_ids[c].data(), chunk_ids[c].size() * 4);
    at += (int64_t)chunk_ids[c].size();
  }
  return LE_OK;
}

}  // extern "C"

// Prefix keys ("virtual ids") on the host, in native code.
//
// The ids must be bit-identical to QwenEdit's multi_turn/cache/keys.py (keys.py:14-58) so both address the same
// cached prefixes:
//   digest(parts...)  = BLAKE2b with a 16-byte digest over, for each part, its length as 8 little-endian bytes
//                       followed by its bytes
//   id(d)             = first 8 digest bytes, little-endian, low 63 bits
//   text id           = id(digest(prev as 8 LE bytes, "t", token as 8 LE signed bytes))          (keys.py:57-58)
//   image block base  = id(digest(prev as 8 LE bytes, "B", content))                             (keys.py:51-54)
//   image block id i  = splitmix64 finaliser of (base + i * 0x9E3779B97F4A7C15), low 63 bits    (keys.py:42-48)
// BLAKE2b follows RFC 7693 (unkeyed, digest length 16, 12 rounds of the G mixing function).
#include <cstdint>
#include <cstring>

#include "qe_common.h"

namespace qe {
namespace {

constexpr uint64_t kIV[8] = {0x6A09E667F3BCC908ull, 0xBB67AE8584CAA73Bull, 0x3C6EF372FE94F82Bull,
                             0xA54FF53A5F1D36F1ull, 0x510E527FADE682D1ull, 0x9B05688C2B3E6C1Full,
                             0x1F83D9ABFB41BD6Bull, 0x5BE0CD19137E2179ull};

constexpr uint8_t kSigma[10][16] = {
    {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15}, {14, 10, 4, 8, 9, 15, 13, 6, 1, 12, 0, 2, 11, 7, 5, 3},
    {11, 8, 12, 0, 5, 2, 15, 13, 10, 14, 3, 6, 7, 1, 9, 4}, {7, 9, 3, 1, 13, 12, 11, 14, 2, 6, 5, 10, 4, 0, 15, 8},
    {9, 0, 5, 7, 2, 4, 10, 15, 14, 1, 11, 12, 6, 8, 3, 13}, {2, 12, 6, 10, 0, 11, 8, 3, 4, 13, 7, 5, 15, 14, 1, 9},
    {12, 5, 1, 15, 14, 13, 4, 10, 0, 7, 6, 3, 9, 2, 8, 11}, {13, 11, 7, 14, 12, 1, 3, 9, 5, 0, 15, 4, 8, 6, 2, 10},
    {6, 15, 14, 9, 11, 3, 0, 8, 12, 2, 13, 7, 1, 4, 10, 5}, {10, 2, 8, 4, 7, 6, 1, 5, 15, 11, 9, 14, 3, 12, 13, 0},
};

inline uint64_t rotr(uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }

inline uint64_t load64(const uint8_t *p) {
  uint64_t v;
  std::memcpy(&v, p, 8);  // little-endian host
  return v;
}

class Blake2b16 {
 public:
  Blake2b16() {
    for (int i = 0; i < 8; ++i) h_[i] = kIV[i];
    h_[0] ^= 0x01010000ull ^ 16ull;  // depth 1, fanout 1, no key, 16-byte digest
  }

  void update(const uint8_t *in, size_t n) {
    while (n > 0) {
      if (fill_ == 128) {  // a full buffer is compressed only once more input follows
        counter_ += 128;
        compress(false);
        fill_ = 0;
      }
      const size_t take = n < 128 - fill_ ? n : 128 - fill_;
      std::memcpy(buf_ + fill_, in, take);
      fill_ += take;
      in += take;
      n -= take;
    }
  }

  // update with a length-prefixed part
  void part(const void *p, size_t n) {
    uint8_t len[8];
    const uint64_t v = n;
    std::memcpy(len, &v, 8);
    update(len, 8);
    update(static_cast<const uint8_t *>(p), n);
  }

  void final16(uint8_t out[16]) {
    counter_ += fill_;
    std::memset(buf_ + fill_, 0, 128 - fill_);
    compress(true);
    std::memcpy(out, h_, 16);
  }

 private:
  void compress(bool last) {
    uint64_t m[16], v[16];
    for (int i = 0; i < 16; ++i) m[i] = load64(buf_ + 8 * i);
    for (int i = 0; i < 8; ++i) {
      v[i] = h_[i];
      v[i + 8] = kIV[i];
    }
    v[12] ^= counter_;  // the high 64 bits of the byte counter stay zero here
    if (last) v[14] = ~v[14];
    for (int r = 0; r < 12; ++r) {
      const uint8_t *s = kSigma[r % 10];
      mix(v, 0, 4, 8, 12, m[s[0]], m[s[1]]);
      mix(v, 1, 5, 9, 13, m[s[2]], m[s[3]]);
      mix(v, 2, 6, 10, 14, m[s[4]], m[s[5]]);
      mix(v, 3, 7, 11, 15, m[s[6]], m[s[7]]);
      mix(v, 0, 5, 10, 15, m[s[8]], m[s[9]]);
      mix(v, 1, 6, 11, 12, m[s[10]], m[s[11]]);
      mix(v, 2, 7, 8, 13, m[s[12]], m[s[13]]);
      mix(v, 3, 4, 9, 14, m[s[14]], m[s[15]]);
    }
    for (int i = 0; i < 8; ++i) h_[i] ^= v[i] ^ v[i + 8];
  }

  static void mix(uint64_t *v, int a, int b, int c, int d, uint64_t x, uint64_t y) {
    v[a] = v[a] + v[b] + x;
    v[d] = rotr(v[d] ^ v[a], 32);
    v[c] = v[c] + v[d];
    v[b] = rotr(v[b] ^ v[c], 24);
    v[a] = v[a] + v[b] + y;
    v[d] = rotr(v[d] ^ v[a], 16);
    v[c] = v[c] + v[d];
    v[b] = rotr(v[b] ^ v[c], 63);
  }

  uint64_t h_[8];
  uint8_t buf_[128] = {};
  size_t fill_ = 0;
  uint64_t counter_ = 0;
};

constexpr uint64_t kMask63 = (1ull << 63) - 1;

inline int64_t digest_id(const uint8_t d[16]) { return int64_t(load64(d) & kMask63); }

inline int64_t text_id(int64_t prev, int64_t token) {
  Blake2b16 h;
  h.part(&prev, 8);
  h.part("t", 1);
  h.part(&token, 8);
  uint8_t d[16];
  h.final16(d);
  return digest_id(d);
}

inline int64_t block_base(int64_t prev, const uint8_t *content, size_t len) {
  Blake2b16 h;
  h.part(&prev, 8);
  h.part("B", 1);
  h.part(content, len);
  uint8_t d[16];
  h.final16(d);
  return digest_id(d);
}

inline int64_t mix63(uint64_t x) {
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x = x ^ (x >> 31);
  return int64_t(x & kMask63);
}

}  // namespace
}  // namespace qe

using qe::fail;

extern "C" {

int qe_blake2b16(const uint8_t *msg, int64_t len, uint8_t *out16) {
  QE_CHECK_ARG(out16 && len >= 0 && (len == 0 || msg), "qe_blake2b16: bad arguments");
  qe::Blake2b16 h;
  h.update(msg, size_t(len));
  h.final16(out16);
  return qe::ok();
}

int qe_keys_text_chain(int64_t prev, const int64_t *tokens, int64_t n, int64_t *out) {
  QE_CHECK_ARG(n >= 0 && (n == 0 || (tokens && out)), "qe_keys_text_chain: bad arguments");
  for (int64_t i = 0; i < n; ++i) {
    prev = qe::text_id(prev, tokens[i]);
    out[i] = prev;
  }
  return qe::ok();
}

int qe_keys_block_ids(int64_t prev, const uint8_t *content, int64_t len, int64_t n, int64_t *out) {
  QE_CHECK_ARG(len >= 0 && n >= 0 && (len == 0 || content) && (n == 0 || out), "qe_keys_block_ids: bad arguments");
  const uint64_t base = uint64_t(qe::block_base(prev, content, size_t(len)));
  for (int64_t i = 0; i < n; ++i) out[i] = qe::mix63(base + uint64_t(i) * 0x9E3779B97F4A7C15ull);
  return qe::ok();
}

}  // extern "C"

// BLAKE3 (plain hash mode, 32-byte output), host code.
//
// The reference fingerprints a byte corpus with the `blake3` crate (crates/sejong-train/src/lib.rs:
// 24-51: a domain string, then per document its length as a little-endian u64 and its bytes); a
// checkpoint carries that fingerprint and a resume is refused when it differs.  This is an own
// implementation of the published BLAKE3 algorithm (compression function of 7 rounds over a 16-word
// state, 1024-byte chunks of 64-byte blocks, chunk chaining values merged in a binary tree whose
// right edge is finished at the end, ROOT flag on the final compression), streaming over the
// caller's parts so that a corpus need not be copied into one buffer.
#include <algorithm>
#include <cstdint>
#include <cstring>

#include "internal.h"

namespace {

constexpr uint32_t kIv[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                             0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
constexpr int kPermutation[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};
constexpr uint32_t kChunkStart = 1, kChunkEnd = 2, kParent = 4, kRoot = 8;
constexpr size_t kBlockLen = 64, kChunkLen = 1024;

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

inline void mix(uint32_t* s, int a, int b, int c, int d, uint32_t x, uint32_t y) {
  s[a] = s[a] + s[b] + x;
  s[d] = rotr(s[d] ^ s[a], 16);
  s[c] = s[c] + s[d];
  s[b] = rotr(s[b] ^ s[c], 12);
  s[a] = s[a] + s[b] + y;
  s[d] = rotr(s[d] ^ s[a], 8);
  s[c] = s[c] + s[d];
  s[b] = rotr(s[b] ^ s[c], 7);
}

// The 16-word compression output for chaining value cv, message block m (16 little-endian words).
void compress(const uint32_t cv[8], const uint32_t m_in[16], uint64_t counter, uint32_t block_len, uint32_t flags,
              uint32_t out[16]) {
  uint32_t s[16] = {cv[0], cv[1], cv[2], cv[3], cv[4], cv[5], cv[6], cv[7],
                    kIv[0], kIv[1], kIv[2], kIv[3], static_cast<uint32_t>(counter),
                    static_cast<uint32_t>(counter >> 32), block_len, flags};
  uint32_t m[16];
  std::memcpy(m, m_in, sizeof(m));
  for (int round = 0; round < 7; ++round) {
    mix(s, 0, 4, 8, 12, m[0], m[1]);
    mix(s, 1, 5, 9, 13, m[2], m[3]);
    mix(s, 2, 6, 10, 14, m[4], m[5]);
    mix(s, 3, 7, 11, 15, m[6], m[7]);
    mix(s, 0, 5, 10, 15, m[8], m[9]);
    mix(s, 1, 6, 11, 12, m[10], m[11]);
    mix(s, 2, 7, 8, 13, m[12], m[13]);
    mix(s, 3, 4, 9, 14, m[14], m[15]);
    if (round < 6) {
      uint32_t p[16];
      for (int i = 0; i < 16; ++i) p[i] = m[kPermutation[i]];
      std::memcpy(m, p, sizeof(m));
    }
  }
  for (int i = 0; i < 8; ++i) {
    out[i] = s[i] ^ s[i + 8];
    out[i + 8] = s[i + 8] ^ cv[i];
  }
}

void words_of(const uint8_t* block, uint32_t w[16]) {
  for (int i = 0; i < 16; ++i)
    w[i] = static_cast<uint32_t>(block[4 * i]) | (static_cast<uint32_t>(block[4 * i + 1]) << 8) |
           (static_cast<uint32_t>(block[4 * i + 2]) << 16) | (static_cast<uint32_t>(block[4 * i + 3]) << 24);
}

// What the final compression of a node needs, kept until it is known whether the node is the root.
struct Output {
  uint32_t cv[8];
  uint32_t block[16];
  uint64_t counter;
  uint32_t block_len, flags;
  void chaining_value(uint32_t out[8]) const {
    uint32_t full[16];
    compress(cv, block, counter, block_len, flags, full);
    std::memcpy(out, full, 32);
  }
};

Output parent_output(const uint32_t left[8], const uint32_t right[8]) {
  Output o;
  std::memcpy(o.cv, kIv, sizeof(o.cv));
  std::memcpy(o.block, left, 32);
  std::memcpy(o.block + 8, right, 32);
  o.counter = 0;
  o.block_len = kBlockLen;
  o.flags = kParent;
  return o;
}

struct Hasher {
  // current chunk
  uint32_t cv[8];
  uint64_t chunk = 0;
  uint8_t buf[kBlockLen];
  size_t buf_len = 0;
  int blocks = 0;  // blocks compressed in the current chunk
  // chaining values of completed subtrees along the left edge (at most 54 for 2^64 bytes)
  uint32_t stack[64][8];
  int depth = 0;

  Hasher() { std::memcpy(cv, kIv, sizeof(cv)); }

  size_t chunk_len() const { return kBlockLen * static_cast<size_t>(blocks) + buf_len; }
  uint32_t start_flag() const { return blocks == 0 ? kChunkStart : 0u; }

  Output chunk_output() const {
    Output o;
    std::memcpy(o.cv, cv, sizeof(o.cv));
    uint8_t block[kBlockLen] = {};
    std::memcpy(block, buf, buf_len);
    words_of(block, o.block);
    o.counter = chunk;
    o.block_len = static_cast<uint32_t>(buf_len);
    o.flags = start_flag() | kChunkEnd;
    return o;
  }

  // A finished chunk's chaining value joins the tree: merge while the chunk count is even.
  void push_chunk_cv(uint32_t chunk_cv[8], uint64_t total_chunks) {
    while ((total_chunks & 1) == 0) {
      --depth;
      uint32_t merged[8];
      parent_output(stack[depth], chunk_cv).chaining_value(merged);
      std::memcpy(chunk_cv, merged, 32);
      total_chunks >>= 1;
    }
    std::memcpy(stack[depth++], chunk_cv, 32);
  }

  void update(const uint8_t* data, size_t len) {
    while (len > 0) {
      if (chunk_len() == kChunkLen) {  // the chunk is complete and more input follows
        uint32_t chunk_cv[8];
        chunk_output().chaining_value(chunk_cv);
        push_chunk_cv(chunk_cv, chunk + 1);
        ++chunk;
        std::memcpy(cv, kIv, sizeof(cv));
        buf_len = 0;
        blocks = 0;
      }
      if (buf_len == kBlockLen) {  // a full block with more input after it: compress it
        uint32_t w[16], full[16];
        words_of(buf, w);
        compress(cv, w, chunk, kBlockLen, start_flag(), full);
        std::memcpy(cv, full, 32);
        ++blocks;
        buf_len = 0;
      }
      const size_t want = std::min(kBlockLen - buf_len, len);
      std::memcpy(buf + buf_len, data, want);
      buf_len += want;
      data += want;
      len -= want;
    }
  }

  void finalize(uint8_t out[32]) const {
    Output o = chunk_output();
    for (int i = depth - 1; i >= 0; --i) {
      uint32_t right[8];
      o.chaining_value(right);
      o = parent_output(stack[i], right);
    }
    uint32_t full[16];
    compress(o.cv, o.block, 0, o.block_len, o.flags | kRoot, full);
    for (int i = 0; i < 8; ++i)
      for (int b = 0; b < 4; ++b) out[4 * i + b] = static_cast<uint8_t>(full[i] >> (8 * b));
  }
};

}  // namespace

extern "C" int sj_blake3(const void* const* parts, const uint64_t* lengths, int count, uint8_t* out) {
  if (count < 0 || (count > 0 && (!parts || !lengths)) || !out)
    return sj::fail(SJ_ERR_ARGUMENT, "sj_blake3: null parts, lengths or output");
  Hasher h;
  for (int i = 0; i < count; ++i) {
    if (lengths[i] && !parts[i]) return sj::fail(SJ_ERR_ARGUMENT, "sj_blake3: part %d is null", i);
    h.update(static_cast<const uint8_t*>(parts[i]), static_cast<size_t>(lengths[i]));
  }
  h.finalize(out);
  return SJ_OK;
}

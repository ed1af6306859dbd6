// Host-side core of the shuffled-epoch token stream (rig/tokens.py:127-272).
//
// The reference walks, per global window ordinal, a keyed 6-round balanced
// Feistel permutation over the next even-bit power-of-two domain with cycle
// walking (rig/tokens.py:136-168), SplitMix64 round keys (:127-133), then a
// binary search over the epoch's shard order (:239-254). That per-row Python
// loop is the data loader's hot spot; here it runs as plain C++ over all rows
// of a local batch: the epoch's window table (per-shard window counts in the
// epoch's shard order), the epoch key and the window copy from the (memory
// mapped) shards into the int32 batch. Only the shard order itself comes from
// the caller, because it is a draw of numpy's PCG64 Generator
// (rig/tokens.py:222-236).
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "../../include/gptb200.h"

static inline uint64_t mix64(uint64_t v) {
  v += 0x9E3779B97F4A7C15ull;
  v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
  v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
  return v ^ (v >> 31);
}

static inline int bit_length(uint64_t x) {
  int n = 0;
  while (x) {
    ++n;
    x >>= 1;
  }
  return n;
}

struct Feistel {
  int half_bits;
  uint64_t half_mask;
  uint64_t round_keys[6];
  Feistel(uint64_t size, uint64_t key) {
    int bits = std::max(2, bit_length(size - 1));
    if (bits % 2) bits += 1;
    half_bits = bits / 2;
    half_mask = (half_bits >= 64) ? ~0ull : ((1ull << half_bits) - 1);
    for (int r = 0; r < 6; ++r) round_keys[r] = mix64(key + (uint64_t)r * 0xD1B54A32D192ED03ull);
  }
  uint64_t apply(uint64_t x) const {
    uint64_t left = x >> half_bits, right = x & half_mask;
    for (int r = 0; r < 6; ++r) {
      uint64_t mixed = mix64(right ^ round_keys[r]) & half_mask;
      uint64_t nl = right;
      right = left ^ mixed;
      left = nl;
    }
    return (left << half_bits) | right;
  }
};

extern "C" uint64_t gptb200_mix_uint64(uint64_t value) { return mix64(value); }

extern "C" uint64_t gptb200_permute_bounded(uint64_t value, uint64_t size, uint64_t key) {
  if (value >= size) return UINT64_MAX;
  if (size == 1) return 0;
  Feistel f(size, key);
  uint64_t c = value;
  for (;;) {
    c = f.apply(c);
    if (c < size) return c;
  }
}

namespace {

// Reads element i of a shard of element type `dtype` (GPTB200_TOKENS_*).
inline int64_t token_at(const void* shard, int dtype, int64_t i) {
  switch (dtype) {
    case GPTB200_TOKENS_U8: return static_cast<const uint8_t*>(shard)[i];
    case GPTB200_TOKENS_U16: return static_cast<const uint16_t*>(shard)[i];
    case GPTB200_TOKENS_I32: return static_cast<const int32_t*>(shard)[i];
    case GPTB200_TOKENS_U32: return static_cast<const uint32_t*>(shard)[i];
    default: return static_cast<const int64_t*>(shard)[i];
  }
}

}  // namespace

extern "C" int gptb200_epoch_windows(const void* const* shards, const int64_t* lengths,
                                     int64_t n_shards, int dtype, const int64_t* order,
                                     int64_t seq_len, uint64_t seed, int64_t epoch,
                                     int64_t first, int64_t rows, int64_t vocab, int32_t* out) {
  if (!shards || !lengths || !order || !out || n_shards <= 0 || seq_len <= 0 || rows < 0 ||
      first < 0 || epoch < 0 || vocab <= 0)
    return GPTB200_EINVAL;
  if (dtype < GPTB200_TOKENS_U8 || dtype > GPTB200_TOKENS_I64) return GPTB200_EINVAL;
  // The epoch's plan: shards visited in `order`, each contributing
  // floor((len - 1) / seq_len) whole windows; ends[j] = windows of the first
  // j + 1 shards of the order.
  std::vector<int64_t> ends(n_shards);
  int64_t total = 0;
  for (int64_t j = 0; j < n_shards; ++j) {
    const int64_t s = order[j];
    if (s < 0 || s >= n_shards) return GPTB200_EINVAL;
    total += std::max<int64_t>(0, (lengths[s] - 1) / seq_len);
    ends[j] = total;
  }
  if (total <= 0 || first + rows > total) return GPTB200_EINVAL;
  const uint64_t size = (uint64_t)total;
  const Feistel f(size, mix64(seed ^ mix64((uint64_t)epoch)));
  int status = GPTB200_OK;
  for (int64_t r = 0; r < rows; ++r) {
    uint64_t w = (uint64_t)(first + r);
    if (size == 1) {
      w = 0;
    } else {
      do w = f.apply(w);
      while (w >= size);  // cycle walking back into [0, size)
    }
    // the shard of the order whose window range holds w
    const int64_t j = std::upper_bound(ends.begin(), ends.end(), (int64_t)w) - ends.begin();
    const int64_t s = order[j];
    const int64_t start = ((int64_t)w - (j ? ends[j - 1] : 0)) * seq_len;
    int32_t* dst = out + r * (seq_len + 1);
    for (int64_t t = 0; t <= seq_len; ++t) {
      const int64_t v = token_at(shards[s], dtype, start + t);
      if (v < 0 || v >= vocab) status = GPTB200_ERANGE;
      dst[t] = (int32_t)v;
    }
  }
  return status;
}

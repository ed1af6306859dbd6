// Host-side core of the shuffled-epoch token stream (rig/tokens.py:127-272).
//
// The reference walks, per global window ordinal, a keyed 6-round balanced
// Feistel permutation over the next even-bit power-of-two domain with cycle
// walking (rig/tokens.py:136-168), SplitMix64 round keys (:127-133), then a
// binary search over the epoch's shard order (:239-254). That per-row Python
// loop is the data loader's hot spot; here it runs as plain C++ over all rows
// of a local batch, and the windows are copied straight from the (memory
// mapped) uint16 shards into the int32 batch. The epoch plan (shard order
// from numpy's Generator, rig/tokens.py:222-236) stays with the Python caller
// because it depends on numpy's PCG64 stream.
#include <stdint.h>
#include <string.h>

#include <algorithm>

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

extern "C" int gptb200_gather_windows(const uint16_t* const* shard_data,
                                      const int64_t* shard_lengths, const int64_t* ordered_shards,
                                      const int64_t* ordered_cumulative, int64_t n_shards,
                                      int64_t windows_per_epoch, uint64_t epoch_key,
                                      int64_t first_epoch_ordinal, int64_t rows, int64_t seq_len,
                                      int64_t vocab, int32_t* out) {
  if (!shard_data || !shard_lengths || !ordered_shards || !ordered_cumulative || !out)
    return GPTB200_EINVAL;
  if (n_shards <= 0 || windows_per_epoch <= 0 || rows < 0 || seq_len <= 0)
    return GPTB200_EINVAL;
  if (first_epoch_ordinal < 0 || first_epoch_ordinal + rows > windows_per_epoch)
    return GPTB200_EINVAL;
  const uint64_t size = (uint64_t)windows_per_epoch;
  Feistel f(size, epoch_key);
  int status = GPTB200_OK;
  for (int64_t r = 0; r < rows; ++r) {
    uint64_t c = (uint64_t)(first_epoch_ordinal + r);
    if (size > 1) {
      do {
        c = f.apply(c);
      } while (c >= size);
    } else {
      c = 0;
    }
    const int64_t permuted = (int64_t)c;
    // searchsorted(cumulative, permuted, side="right")
    const int64_t* it =
        std::upper_bound(ordered_cumulative, ordered_cumulative + n_shards, permuted);
    const int64_t oi = it - ordered_cumulative;
    if (oi >= n_shards) return GPTB200_EINVAL;
    const int64_t prev = oi ? ordered_cumulative[oi - 1] : 0;
    const int64_t shard = ordered_shards[oi];
    const int64_t start = (permuted - prev) * seq_len;
    if (start + seq_len + 1 > shard_lengths[shard]) return GPTB200_EINVAL;
    const uint16_t* src = shard_data[shard] + start;
    int32_t* dst = out + r * (seq_len + 1);
    for (int64_t t = 0; t <= seq_len; ++t) {
      const int32_t v = (int32_t)src[t];
      if (v >= vocab) status = GPTB200_ERANGE;
      dst[t] = v;
    }
  }
  return status;
}

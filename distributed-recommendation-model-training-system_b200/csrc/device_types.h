// device_types.h -- plain structs shared by the host runtime and the sm_100a kernels.
//
// HBM layout of one table shard (dense, direct-mapped):
//   state   : float[rows][3][D]   row = [w(D) | m(D) | v(D)], the reference's row
//             layout (src/store/shard_store.cpp:21-29), 12*D bytes per row
//   updates : uint64[rows]        row_updates counter (RowState::row_updates)
// A key k lives on shard k % shard_count at slot k / shard_count
// (src/access/prepared_lookup.cpp:54, src/store/shard_store.cpp:77).
#pragma once
#include <stdint.h>

namespace eps_b200 {

// Device-resident optimizer bookkeeping of one table (TableState,
// src/store/shard_store.hpp:11-16).  Kept on the GPU so that a rejected Push
// (decided on the device) never advances the host's view of beta powers.
struct DeviceTable {
  float beta1_power;
  float beta2_power;
  unsigned long long optimizer_sequence;
  // Upper bound of |w|, |m| and v over every row ever written (float bits).
  // Used to prove that an update cannot overflow (see push kernels).
  unsigned int state_absmax_bits;
  unsigned int pad;
};

// The id -> slot index of a hashed table (any u64 key; a row is created on its
// first touch, as ShardStore::Ensure does, src/store/shard_store.cpp:76-115):
// open addressing with linear probing over `mask + 1` entries (at most half
// full), a key entry claimed by one compare-and-swap; the winner takes the next
// slot and writes the row's initial value.  Device-resident, one per table.
struct HashIndex {
  unsigned long long* keys;         // [mask + 1], kEmptyKey = free (key ~0 uses `top`)
  unsigned int* slots;              // [mask + 2] slot of each entry (entry mask + 1: key ~0)
  unsigned long long* slot_keys;    // [capacity] key of each slot
  unsigned long long* used;         // slots handed out (may pass capacity: those failed)
  unsigned int* top;                // entry of key ~0 claimed
  unsigned long long mask;
  unsigned long long capacity;
  // the row initializer (shard_store.cpp:104-111)
  float* state;
  unsigned long long* updates;
  unsigned int dim, table_id;
  unsigned long long seed;
  float init_min, init_max;
  int has_bounds;
  float bound_min, bound_max;
};
constexpr unsigned long long kEmptyKey = ~0ull;
constexpr unsigned int kNoSlot = 0xFFFFFFFFu;       // entry without a usable slot

// One table as seen by a Push: constant optimizer parameters plus pointers.
struct PushTable {
  float* state;
  unsigned long long* updates;
  DeviceTable* dtable;
  unsigned long long rows;
  unsigned long long occurrences;   // occurrences of this table in the lookup
  float learning_rate, beta1, beta2, epsilon;
  float one_minus_beta1, one_minus_beta2;
  float bound_min, bound_max;
  int has_bounds;
  unsigned int dim;
  float lr_t;                       // bias-corrected rate, written on the device
  unsigned int pad;
};

// One feature of a lookup.  `item` = one bag (for sequence features the bag
// structure is kept; every position is its own output row).
struct LookupFeature {
  const unsigned long long* keys;
  const unsigned long long* offsets;
  const unsigned long long* lengths;  // original bag lengths, or null => offset diffs
  float* out;
  const float* state;
  unsigned long long rows;             // slots of the table on this shard
  unsigned long long key_count;
  unsigned long long bag_count;
  unsigned long long bag_base;         // prefix of bags over features
  unsigned long long occ_base;         // first occurrence index in the ticket
  unsigned long long scale_base;       // first gradient-row index in row_scale
  unsigned int dim;
  unsigned int pooling;                // 0 sum, 1 mean, 2 sequence
  unsigned int table_rank;             // rank of the table inside this lookup
  unsigned int feature_index;          // index inside the lookup (gradient slot)
  unsigned int has_padding;            // keys equal to padding_key are dropped
  unsigned int unit_bags;              // bags per work unit (pooled features)
  unsigned long long padding_key;
  // work units of the emit and gather kernels: unit_bags consecutive bags of a
  // pooled feature, or kUnitPositions consecutive positions (and the same span
  // of offsets, which the unit validates) of a sequence feature
  unsigned long long unit_base;        // prefix of units over features
  unsigned long long units;
  // the emit kernel's units: always kUnitBags bags (or kUnitPositions positions)
  unsigned long long emit_base;
  unsigned long long emit_units;
  // hashed table: slots[i] is occurrence i's resolved slot (kPadSlot: padding,
  // kNoSlot: not resolved -- another shard's key or the table is full)
  const HashIndex* hash;
  const unsigned int* slots;
};
constexpr unsigned int kPadSlot = 0xFFFFFFFEu;   // slot marker of a padding key
constexpr unsigned int kUnitBags = 8;
constexpr unsigned int kUnitPositions = 256;
constexpr unsigned int kUnitSlices = kUnitPositions / 32;   // 32-position slices of a unit

constexpr unsigned int kEmitShortBags = 32;

// Bags per gather unit of a pooled feature: one bag when bags hold 8 or more
// keys on average (enough work and parallelism per bag), else `group` bags (the
// gather's lanes per group, 8..32: a lane holds one bag's range), whose keys the
// group walks as one run, so that the chain of dependent loads (offsets, keys,
// rows) is paid once per unit and rows load back to back across bags.
inline unsigned feature_unit_bags(unsigned pooling, unsigned long long key_count,
                                  unsigned long long bag_count, unsigned group) {
  if (pooling == 2) return 0;
  if (bag_count && key_count >= 8ull * bag_count) return 1u;
  return group < kUnitBags ? kUnitBags : (group > 32u ? 32u : group);
}

// Bags per emit unit of a pooled feature (one warp per unit, one occurrence per
// lane and step): kUnitBags for long bags (8 or more keys on average),
// kEmitShortBags for short ones, so a step of one-key bags still fills the warp.
#ifdef __CUDACC__
__host__ __device__
#endif
inline unsigned emit_unit_bags(unsigned long long key_count, unsigned long long bag_count) {
  return (bag_count && key_count >= 8ull * bag_count) ? kUnitBags : kEmitShortBags;
}

// Work units of one feature (see LookupFeature::units); `unit_bags` bags per
// unit of a pooled feature.
inline unsigned long long feature_units(unsigned pooling, unsigned long long key_count,
                                        unsigned long long bag_count, unsigned unit_bags) {
  if (pooling != 2) return (bag_count + unit_bags - 1) / unit_bags;
  const unsigned long long by_keys = (key_count + kUnitPositions - 1) / kUnitPositions;
  if (bag_count == 0) return by_keys;
  const unsigned long long by_offsets = (bag_count + 1 + kUnitPositions - 1) / kUnitPositions;
  return by_keys > by_offsets ? by_keys : by_offsets;
}

// Gradient source of one feature for a Push.
struct PushFeature {
  const float* grad;                   // [rows][dim]
  unsigned long long rows;
  unsigned long long scale_base;
  unsigned int dim;
  unsigned int table_rank;
};

enum PushMode : unsigned int { kModeSafe = 0, kModeChecked = 1, kModeRejected = 2 };
enum RejectBits : unsigned int {
  kRejectNonFiniteInput = 1u,   // src/access/batch_access.cpp:97
  kRejectLearningRate = 2u,     // src/update/lazy_adam.cpp:12
  kRejectReduction = 4u,        // src/access/batch_access.cpp:122-123
  kRejectOptimizer = 8u,        // src/update/lazy_adam.cpp:20-21
};
enum LookupErrorBits : unsigned int {
  kLookupBadOffsets = 1u,       // src/access/batch_access.cpp:14-16
  kLookupBadKey = 2u,           // key routed to another shard / outside the table
  kLookupShortLength = 4u,      // src/access/batch_access.cpp:18-20
  kLookupSortFailed = 8u,       // a coalescing-sort wait ran out (never expected)
  kLookupCapacity = 64u,        // a hashed table holds its capacity of rows already
};

// Per-push control block (device).  Zeroed before each push.
struct PushControl {
  unsigned int nonfinite;
  unsigned int maxabs_bits;
  unsigned int mode;
  unsigned int reject_bits;
  unsigned int long_count;
  unsigned int blocks_done;
  unsigned int accepted;
  unsigned int piece_count;     // pieces reserved by long rows
  unsigned int blocks_done_b;   // blocks of push stage B that finished
  unsigned int blocks_done_c;   // blocks of push stage C that finished
  unsigned int work_a;          // chunks claimed in push stage A
  unsigned int work_b;          // row chunks claimed in push stage B
  unsigned int work_long;       // long rows claimed in push stage B
  unsigned int work_ring;       // row chunks claimed by the async-ring row kernel
};

// A long coalesced row (more than kLongRun occurrences): its occurrences are
// reduced in pieces of kPiece into part[piece_base ..] and combined in piece
// order by the long-row kernel.
struct LongRecord {
  unsigned long long key;       // composite (table rank, slot)
  unsigned int piece_base;
  unsigned int npieces;
};

// One coalesced row of a lookup ticket (rows[u] for run u of the sorted keys),
// prepared on the side stream after the coalescing sort so that the push reads
// everything it needs about a row in one 16-byte load:
//   b < 2^31  -- a single-occurrence row: a = its gradient source, b = the
//                float bits of its row scale (positive);
//   b = 2^31 | len, len in 2..long_run -- a = the piece that reduces all of
//                its occurrences in order (its gradient is part[a]);
//   b = kRowSkip -- a padding row or a long row (handled by pieces).
struct alignas(16) RowRec {
  unsigned long long key;       // composite (table rank, slot)
  unsigned int a, b;
};
constexpr unsigned int kRowMulti = 0x80000000u;
constexpr unsigned int kRowSkip = 0xFFFFFFFFu;
// Counts of the row plan: `piece_count` pieces (one per row with 2..long_run
// occurrences, ceil(len / kPiece) per long row) and `long_count` LongRecords.
struct RowPlan {
  unsigned int long_count, piece_count, reserved0, reserved1;
};

constexpr int kLongRun = 64;    // rows with more occurrences than this are "long"
#ifndef EPS_PIECE
#define EPS_PIECE 64
#endif
constexpr int kPiece = EPS_PIECE;   // occurrences per piece of a long row
constexpr unsigned int kMaxFeatures = 1024;
constexpr unsigned int kRowBits = 22;   // gradient row bits in the source code

}  // namespace eps_b200

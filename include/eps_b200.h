/*
 * eps_b200.h -- C ABI of the B200 embedding parameter store (libeps_b200.so).
 *
 * The library keeps embedding tables and their sparse LazyAdam state resident in
 * GPU memory and runs the reference parameter server's hot path on the GPU:
 * batched pull (gather + sum/mean/sequence pooling), push (coalesce duplicate ids,
 * segment-sum their gradients) and the row-wise LazyAdam update.
 *
 * Citations name the interface of the reference project
 * (Zhang-Xin-Duke/distributed-recommendation-model-training-system) that each
 * entry point replaces, as path:line inside that project.
 *
 * Conventions (mirroring include/eps/runtime_c.h and adapters/entropy/runtime_c.cpp):
 *  - every entry point returns 0 on success, else eps::Error::Code + 1
 *    (include/eps/types.hpp:17-25) and copies the message into status->message;
 *  - plain pointers and sizes only; buffers flagged `device >= 0` / `*_on_device`
 *    are device pointers on the store's GPU, otherwise host pointers;
 *  - `stream` is a cudaStream_t (NULL = the store's own stream, a blocking stream
 *    ordered with the legacy default stream).  All work of one
 *    store is serialised; calls on one store are thread-safe (one mutex, as the
 *    reference runtime's per-runtime mutex, adapters/entropy/runtime_c.cpp:177).
 *  - nothing here allocates on the caller's behalf except the returned store;
 *    results are written into caller-provided buffers.
 */
#ifndef EPS_B200_H
#define EPS_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EPS_B200_ABI 3

#if defined(_WIN32)
#define EPS_B200_EXPORT __declspec(dllexport)
#else
#define EPS_B200_EXPORT __attribute__((visibility("default")))
#endif

/* Same layout and codes as EpsStatus (include/eps/runtime_c.h:8). */
typedef struct { int32_t code; char message[1024]; } EpsB200Status;

enum {
  EPS_B200_OK = 0,
  EPS_B200_INVALID_ARGUMENT = 1,   /* Error::Code::invalid_argument + 1 */
  EPS_B200_UNAVAILABLE = 2,
  EPS_B200_STALE_GENERATION = 3,
  EPS_B200_RETIRED_REQUEST = 4,
  EPS_B200_CAPACITY_EXCEEDED = 5,
  EPS_B200_RUN_FAILED = 6
};

/* eps::Pooling (include/eps/types.hpp:51) */
enum { EPS_B200_SUM = 0, EPS_B200_MEAN = 1, EPS_B200_SEQUENCE = 2 };

typedef struct EpsB200Store EpsB200Store;

/* Subset of eps::RuntimeOptions (include/eps/runtime.hpp:15-39) plus the GPU. */
typedef struct {
  int32_t device;
  uint32_t shard_id;
  uint32_t shard_count;
  uint32_t max_live_tickets;     /* RuntimeOptions::max_live_tickets (runtime.hpp:24) */
  uint64_t partition_epoch;
  uint64_t state_bytes;          /* HBM budget for table state (runtime.hpp:20) */
  uint32_t flags;                /* EPS_B200_FLAG_* */
  /* Pushes left enqueued (wait == 0) before the next lookup waits for the
   * oldest: bounds the ticket memory of a caller that runs ahead of the device
   * (each enqueued push keeps its lookup's slab).  0 = 16. */
  uint32_t max_enqueued_pushes;
} EpsB200Options;

/* Sum every coalesced row's gradients serially in occurrence order, as the
 * reference does (src/access/batch_access.cpp:109-119), also for rows with very
 * many occurrences.  Without it such rows (> 64 occurrences) are reduced in
 * parallel pieces combined in a fixed order: deterministic, and within 1e-6
 * relative of the serial sum, but not bit-identical. */
#define EPS_B200_FLAG_REFERENCE_ORDER 1u

/* Update coalesced rows with the register-resident kernels only.  By default a
 * push whose tables all have one dimension in {32, 64, 128} (16-byte aligned
 * gradients) streams its rows through a shared-memory ring of asynchronous
 * copies; other pushes always take the register path.  Both give identical
 * results; the flag exists so that tests can run the second path on any shape. */
#define EPS_B200_FLAG_REGISTER_ROWS 2u

/* eps::TableDefinition + eps::OptimizerConfig (include/eps/types.hpp:76-97).
 * key_space > 0: a dense table -- keys lie in [0, key_space); the shard holds the
 * slots of keys k with k % shard_count == shard_id (src/store/shard_store.cpp:77),
 * at slot k / shard_count, initialised up front with the reference initializer.
 * key_space == 0: a hashed table -- any 64-bit key owned by the shard; a row is
 * created on the key's first touch (any lookup, read_state or load_state), with
 * the same initializer, as ShardStore::Ensure does (src/store/shard_store.cpp:
 * 76-115); the shard holds at most `capacity` rows (then lookups of unseen keys
 * fail with "hashed table capacity exceeded").  An open-addressing index of
 * 2 x capacity entries (rounded up to a power of two) maps keys to rows. */
typedef struct {
  uint32_t id;
  uint32_t dimension;
  uint32_t shard_count;
  int32_t has_weight_bounds;
  uint64_t partition_epoch;
  float learning_rate, beta1, beta2, epsilon;
  float initial_beta1_power, initial_beta2_power;
  float weight_min, weight_max;
  float initialization_min, initialization_max;
  uint64_t initialization_seed;
  uint64_t key_space;
  uint64_t capacity;             /* hashed tables (key_space == 0): rows on this shard */
} EpsB200Table;

/* eps::FeatureInput (include/eps/types.hpp:99-107).  valid_lengths may be NULL
 * (then the offset differences are the bag lengths).  has_padding / padding_key
 * as eps::entropy::Feature::padding_key (include/eps/entropy_adapter.hpp:13,
 * EpsFeature in include/eps/runtime_c.h:10-15): keys equal to padding_key are
 * dropped as in PrepareAdapterInput (src/access/prepare_queue.cpp:58-85) --
 * pooled bags sum the other keys and mean divides by their count; sequence
 * outputs keep every position, padding positions read 0 and take no gradient.
 * With has_padding, valid_lengths must be NULL (the kept counts are the
 * lengths).  The multi-GPU round takes padding keys too: they go to no shard,
 * and every shard receives the kept counts as the bags' valid lengths. */
typedef struct {
  uint32_t table, feature, pooling, has_padding;
  const uint64_t* keys; uint64_t key_count;
  const uint64_t* offsets; uint64_t offset_count;
  const uint64_t* valid_lengths;
  uint64_t padding_key;
} EpsB200Feature;

/* Feature tensor [rows, columns] f32: eps::EpsBuffer (include/eps/runtime_c.h:14-19)
 * without the ownership callbacks, since the caller owns every buffer. */
typedef struct {
  uint32_t feature, reserved;
  uint64_t rows, columns;
  void* data;
  int32_t device;                /* < 0: host memory */
  int32_t reserved2;
} EpsB200Buffer;

/* Counters in the spirit of eps::RuntimeStats (include/eps/runtime.hpp:48-95). */
typedef struct {
  uint64_t lookups, updates, rejected_updates, duplicate_requests;
  uint64_t live_tickets, state_bytes, rows, tables;
  uint64_t kernel_launches;      /* device kernels this store has launched */
} EpsB200Stats;

/* Phases of a lookup + push round, for eps_b200_profile. */
enum {
  EPS_B200_PHASE_LOOKUP = 0,     /* gather + pooling */
  EPS_B200_PHASE_SORT = 1,       /* stable radix sort, segments and row plan */
  EPS_B200_PHASE_PRESCAN = 2,    /* gradient finiteness / bound scan + decision */
  EPS_B200_PHASE_APPLY = 3,      /* LazyAdam row updates (single rows and piece sums) */
  EPS_B200_PHASE_FINALIZE = 4,   /* beta powers / optimizer sequence (own launch only
                                    for a push without occurrences) */
  EPS_B200_PHASE_EMIT = 5,       /* occurrence list of a lookup that will be pushed */
  EPS_B200_PHASE_PIECES = 6,     /* in-order piece sums of rows with several occurrences */
  EPS_B200_PHASE_LONG = 7,       /* long rows (piece combine + LazyAdam), checked apply */
  EPS_B200_PHASES = 8
};

EPS_B200_EXPORT uint32_t eps_b200_abi_version(void);

/* Creates one shard store on `device`.  Replaces constructing
 * eps::CpuParameterService (include/eps/runtime.hpp:104) /
 * eps::CudaCacheBackend (include/eps/cuda_cache_backend.hpp:19). */
EPS_B200_EXPORT int eps_b200_create(const EpsB200Options* options, EpsB200Store** out, EpsB200Status* status);
/* Waits for the store's work (its own completion event, recorded after every
 * call on whatever stream the call ran on, and its own streams), then frees it.
 * No caller stream is used, so callers may destroy their streams first. */
EPS_B200_EXPORT void eps_b200_destroy(EpsB200Store* store);

/* ParameterService::CreateTable (include/eps/parameter_service.hpp:16),
 * CacheBackend::Define (include/eps/cache_backend.hpp:15); validation of
 * ShardStore::Create (src/store/shard_store.cpp:33-60).  Idempotent for an
 * identical definition. */
EPS_B200_EXPORT int eps_b200_create_table(EpsB200Store* store, const EpsB200Table* table,
                          EpsB200Status* status);

/* Pull.  With shard_partial == 0: DistributedClient::Lookup
 * (include/eps/distributed_client.hpp:36) over this store -- pooled outputs
 * are merged and mean bags divided by the bag length
 * (src/client/distributed_client.cpp:173-188,227-232).  With shard_partial == 1:
 * ParameterService::Lookup (include/eps/parameter_service.hpp:17) -- the
 * unnormalised shard contribution of src/access/batch_access.cpp:53-80 for keys
 * owned by this shard, valid_lengths carrying the original bag lengths.
 * outputs[i] receives feature i: [bags, dim] (sum/mean) or [keys, dim]
 * (sequence).  Unless read_only, *ticket receives the lookup ticket to pass to
 * eps_b200_push or eps_b200_release (LookupReply::ticket, types.hpp:151-156).
 * Device inputs are validated on the GPU; such errors are reported by the next
 * push / release / synchronize of the ticket.  Host outputs imply a synchronous
 * call that reports them directly.  outputs == NULL (read_only == 0 only) is a
 * push-only lookup: the ticket's occurrence list and coalescing sort are built,
 * nothing is gathered -- for a caller that pushes gradients of rows it already
 * holds (the Lookup + Push of a push-heavy round, whose Push alone is timed).
 * Likewise, with read_only == 0, a single output whose data is NULL makes that
 * feature push-only (its layout fields are still checked). */
EPS_B200_EXPORT int eps_b200_lookup(EpsB200Store* store, const EpsB200Feature* features, uint64_t count,
                    int32_t input_on_device, int32_t read_only, int32_t shard_partial,
                    EpsB200Buffer* outputs, void* stream, uint64_t* ticket,
                    EpsB200Status* status);

/* Read-only pooled lookup that allocates no device memory.  It has no
 * counterpart in the reference.  It gives the same outputs as eps_b200_lookup
 * with read_only = 1 and shard_partial = 0 for device inputs and device
 * outputs, for callers that must not allocate while serving a request (an
 * inference engine or framework that owns all GPU memory through its own pool,
 * or a latency-critical loop that must never wait on an allocator).
 * Limits and sharing:
 *  - 1 to 256 features per call (larger counts fail with CAPACITY_EXCEEDED);
 *    inputs and outputs must be device buffers on the store's GPU; every
 *    feature must read a dense table (key_space > 0): a hashed table's rows are
 *    found through per-call slot lists, which would need device memory;
 *  - the feature descriptors go to one fixed ~42 KiB array per GPU, created when
 *    the library is loaded on that GPU and kept until the process exits; every
 *    call on that GPU reuses it.  The calls of one store are ordered on the GPU
 *    whatever their streams, so only calls of different stores on one GPU (or of
 *    other users of the library in the process) can overlap, and those race;
 *  - the descriptors are handed to the GPU as kernel parameters, so the caller's
 *    `features` array may be reused as soon as the call returns;
 *  - the first call on a GPU looks up that array's device address (cached for
 *    the life of the process), so make the first call before any CUDA stream
 *    capture starts;
 *  - invalid keys or offsets are reported by the next eps_b200_synchronize. */
EPS_B200_EXPORT int eps_b200_lookup_noalloc(EpsB200Store* store, const EpsB200Feature* features,
                                            uint64_t count, EpsB200Buffer* outputs, void* stream,
                                            EpsB200Status* status);

/* Push gradients of a ticket's feature tensors: DistributedClient::Push /
 * ParameterService::Push (include/eps/parameter_service.hpp:18), i.e.
 * ReduceGradients (src/access/batch_access.cpp:82-125) + ValidateLazyAdam /
 * ApplyLazyAdam (src/update/lazy_adam.cpp:7-42), all-or-nothing.  A rejected
 * push leaves the state unchanged and the ticket live (retryable); a push of an
 * already completed ticket is acknowledged without effect.  wait == 0 returns
 * after enqueueing; its outcome is then reported by eps_b200_synchronize. */
EPS_B200_EXPORT int eps_b200_push(EpsB200Store* store, uint64_t ticket, const EpsB200Buffer* gradients,
                  uint64_t count, void* stream, int32_t wait, EpsB200Status* status);

/* ParameterService::Release (include/eps/parameter_service.hpp:20). */
EPS_B200_EXPORT int eps_b200_release(EpsB200Store* store, uint64_t ticket, EpsB200Status* status);

/* The coalesced rows of a lookup ticket -- what a Push reduces -- as the
 * reference's CompactGradients CSR (BuildCompactGradients,
 * src/access/compact_gradients.cpp:41-72; ReduceGradients' unique rows and their
 * ordered occurrences, src/access/batch_access.cpp:99-121): per unique row its
 * table id and key, row_offsets[rows + 1] into the references, and per reference
 * (in the order the row's gradients are summed) the feature id, the gradient row
 * (bag, or position for sequence features) and its scale (1/length for mean).
 * Rows come in ascending (table, key) order; the reference lists them in first
 * occurrence order, which no result depends on.  Waits for the ticket's lookup.
 * *rows_out / *references_out always receive the counts; with tables == NULL
 * nothing else is written. */
EPS_B200_EXPORT int eps_b200_ticket_coalesced(EpsB200Store* store, uint64_t ticket, uint32_t* tables,
                                              uint64_t* keys, uint64_t* row_offsets,
                                              uint32_t* features, uint64_t* sources, float* scales,
                                              uint64_t row_capacity, uint64_t reference_capacity,
                                              uint64_t* rows_out, uint64_t* references_out,
                                              EpsB200Status* status);

/* Waits for all queued work and reports the first deferred error
 * (DeviceTensor::WaitOnStream contract, include/eps/cache_agent.hpp:7-14). */
EPS_B200_EXPORT int eps_b200_synchronize(EpsB200Store* store, EpsB200Status* status);

/* ParameterService::ReadState (include/eps/parameter_service.hpp:23-24) /
 * CacheBackend::ReadBack (include/eps/cache_backend.hpp:27): host arrays,
 * weights/first/second are [count, dim]. */
EPS_B200_EXPORT int eps_b200_read_state(EpsB200Store* store, uint32_t table, const uint64_t* keys,
                        uint64_t count, float* weights, float* first, float* second,
                        uint64_t* row_updates, EpsB200Status* status);

/* CacheBackend::Load (include/eps/cache_backend.hpp:17-18) /
 * ShardStore::Import (src/store/shard_store.cpp:126-137): overwrite rows with
 * finite state, v >= 0 (src/cache/host_backend.cpp:135-140). */
EPS_B200_EXPORT int eps_b200_load_state(EpsB200Store* store, uint32_t table, const uint64_t* keys,
                        uint64_t count, const float* weights, const float* first,
                        const float* second, const uint64_t* row_updates,
                        EpsB200Status* status);

/* The table's optimizer bookkeeping (TableState, src/store/shard_store.hpp:11-16;
 * the values an UpdateContext carries, include/eps/types.hpp:180-188). */
EPS_B200_EXPORT int eps_b200_optimizer_state(EpsB200Store* store, uint32_t table, uint64_t* optimizer_sequence,
                             float* beta1_power, float* beta2_power, EpsB200Status* status);

/* Per-phase device time measured with CUDA events recorded on the launching
 * stream around each phase (the reference's PhaseTimer counters,
 * src/common/phase_timer.hpp:9-23, RuntimeStats *_nanoseconds fields).
 * mode 1: reset and start recording, 0: stop, -1: leave as is.  Each output
 * array (may be NULL) has EPS_B200_PHASES entries: accumulated milliseconds,
 * kernel launches and calls per phase, collected after the recorded work ends. */
EPS_B200_EXPORT int eps_b200_profile(EpsB200Store* store, int32_t mode, double* phase_ms,
                                     uint64_t* phase_launches, uint64_t* phase_calls,
                                     EpsB200Status* status);

/* ---- Multi-GPU round: the client side of a sharded lookup / push.
 * A route splits device-resident features over `shard_count` shards (one per
 * GPU; 1 .. 32, shards x features <= 1024) by key % shard_count:
 *   PrepareLookupInputs (src/access/prepared_lookup.cpp:47-83) on the device.
 * Shard o's part of feature f keeps the bags that have keys on o, with the
 * original (global) bag lengths as valid lengths, so the shard's
 * eps_b200_lookup(shard_partial = 1) returns the reference's shard contribution
 * for exactly those bags (bags without keys there contribute zeros).
 * Asynchronous: `counts` (device, int64 [shard_count][5 * count + 1]) receives,
 * for every shard o, the row sent to o before the payload: (keys, kept bags)
 * of every feature, then the features' table ids, then their poolings, then
 * their distinct keys U, then the input-error bits (nonzero: offsets not
 * monotone from 0 to key_count, a valid length that differs from the offset
 * difference, or a key >= the table's key_space).  U > 0 marks a deduplicated
 * group: feature f of a dense table whose kept bags on o hold one key each (or
 * a sequence feature), with U distinct keys among its keys (U < keys).  Its
 * owner returns each distinct row once (U partial rows) and the merge reads a
 * bag's row by its key's rank; the values and their order of addition are
 * those of the per-bag partials.  Gradients are not deduplicated.  The inputs
 * must stay valid until eps_b200_route_release. */
EPS_B200_EXPORT int eps_b200_route(EpsB200Store* store, const EpsB200Feature* features, uint64_t count,
                                   uint32_t shard_count, void* stream, uint64_t* route,
                                   int64_t* counts, EpsB200Status* status);
/* Writes the u64 words sent to every shard, shard after shard (what the
 * reference's DistributedClient sends in each shard's LookupRequest,
 * src/client/distributed_client.cpp:96-104): for shard o, the keys of every
 * feature, then every feature's kept-bag offsets (kept + 1 words), then every
 * feature's kept-bag valid lengths, then for every deduplicated feature
 * [0, U, its U distinct keys] (the offsets and keys of one sequence bag).
 * Shard o's part has sum_f (keys + 2 * kept + 1 + (U ? U + 2 : 0)) words. */
EPS_B200_EXPORT int eps_b200_route_scatter(EpsB200Store* store, uint64_t route, uint64_t* payload,
                                           void* stream, EpsB200Status* status);
/* Client merge (src/client/distributed_client.cpp:173-188,227-232): partials holds the
 * shard contributions received from every shard, shard after shard, each
 * feature after feature as [kept bags, dim] (sum/mean), [keys, dim]
 * (sequence) or [U, dim] (deduplicated: the distinct rows); outputs[i] ([bags, dim] or [keys, dim], device) receives the
 * zero-initialised shard-ordered sum, mean bags divided by (float)length, and
 * sequence rows at their positions. */
EPS_B200_EXPORT int eps_b200_route_merge(EpsB200Store* store, uint64_t route, const float* partials,
                                         const EpsB200Buffer* outputs, void* stream,
                                         EpsB200Status* status);
/* Push split (src/client/distributed_client.cpp:252-265): gathers into `send`
 * (device, the layout of route_merge's partials) the gradient rows each shard
 * needs: the kept bags' rows of pooled features, the keys' rows of sequence
 * features (deduplicated groups too), shard after shard, feature after feature.
 * If `nonfinite` (device u32[2], may be NULL) is given, 1 is stored in [0] when
 * any value of any gradient tensor is not finite (the client check of
 * src/client/distributed_client.cpp:249) and the largest |value| (float bits)
 * is max-ed into [1]; the caller zeroes both. */
EPS_B200_EXPORT int eps_b200_route_gather(EpsB200Store* store, uint64_t route,
                                          const EpsB200Buffer* gradients, float* send,
                                          uint32_t* nonfinite, void* stream, EpsB200Status* status);
/* Owner side of a sharded round: ParameterService::Lookup of the combined
 * request of `requesters` clients (include/eps/parameter_service.hpp:17).
 * payload (device) holds the words every requester's route_scatter sent to this
 * shard, requester after requester; peer_counts (host, [requesters][F][3]) the
 * (keys, kept bags, distinct keys U) of each part; tables / poolings (host,
 * [F]) the feature schema shared by all requesters.  Runs
 * eps_b200_lookup(shard_partial = 1) on the requesters' features (ids r * F +
 * f), writing the contributions into `partials` (device), requester after
 * requester, feature after feature, as [kept bags, dim] (sum/mean), [keys, dim]
 * (sequence) or, for a deduplicated part (U > 0), [U, dim]: the rows of its
 * distinct keys, gathered by a read-only lookup while the ticketed lookup only
 * lists the part's occurrences.  *ticket as for eps_b200_lookup. */
EPS_B200_EXPORT int eps_b200_serve(EpsB200Store* store, const uint64_t* payload,
                                   const uint64_t* peer_counts, const uint32_t* tables,
                                   const uint32_t* poolings, uint32_t requesters,
                                   uint32_t feature_count, int32_t read_only, float* partials,
                                   void* stream, uint64_t* ticket, EpsB200Status* status);
/* Owner side of the push of a served round (ParameterService::Push,
 * include/eps/parameter_service.hpp:18): gradients (device) hold the rows every
 * requester's route_gather sent: one row per kept bag (sum/mean) or key
 * (sequence) of every part, requester after requester, feature after feature;
 * peer_counts as for eps_b200_serve.
 * `reject` (device u32[2], may be NULL): the requesters' route_gather words
 * max-reduced over every rank.  If [0] is nonzero when the push runs, the push
 * is rejected on the device as a non-finite input (state unchanged, ticket
 * live); [1], an upper bound of every |g| of the round, then replaces the
 * push's own scan of the gradients in its overflow check.  With wait == 0 the
 * outcome is reported by eps_b200_synchronize. */
EPS_B200_EXPORT int eps_b200_serve_push(EpsB200Store* store, uint64_t ticket, const float* gradients,
                                        const uint64_t* peer_counts, const uint32_t* tables,
                                        const uint32_t* poolings, uint32_t requesters,
                                        uint32_t feature_count, const uint32_t* reject,
                                        void* stream, int32_t wait, EpsB200Status* status);
/* Frees a route (after the work that uses it has been enqueued). */
EPS_B200_EXPORT int eps_b200_route_release(EpsB200Store* store, uint64_t route, EpsB200Status* status);

/* ---- Exchange of a multi-GPU round (no counterpart in the reference, whose
 * shards talk over BRPC): an NCCL communicator over the round's ranks, one per
 * GPU, whose calls enqueue NCCL group send/receive straight onto the caller's
 * stream.  NCCL is loaded at run time (libnccl.so.2); without it these calls
 * fail with EPS_B200_UNAVAILABLE.  The 128-byte unique id is made by one rank
 * and handed to all ranks (e.g. over torch.distributed). */
typedef struct EpsB200Comm EpsB200Comm;
EPS_B200_EXPORT int eps_b200_comm_unique_id(uint8_t* id, EpsB200Status* status);
EPS_B200_EXPORT int eps_b200_comm_create(int32_t device, uint32_t rank, uint32_t world,
                                         const uint8_t* id, EpsB200Comm** out,
                                         EpsB200Status* status);
EPS_B200_EXPORT void eps_b200_comm_destroy(EpsB200Comm* comm);
/* All-to-all with per-peer element counts (send_counts / recv_counts: host,
 * [world]); peer p's block starts after the blocks of peers 0 .. p-1. */
EPS_B200_EXPORT int eps_b200_comm_alltoallv(EpsB200Comm* comm, const void* send,
                                            const uint64_t* send_counts, void* recv,
                                            const uint64_t* recv_counts, uint32_t elem_bytes,
                                            void* stream, EpsB200Status* status);
/* In-place element-wise maximum of `count` u32 over all ranks. */
EPS_B200_EXPORT int eps_b200_comm_allreduce_max(EpsB200Comm* comm, uint32_t* buf, uint64_t count,
                                                void* stream, EpsB200Status* status);

/* ---- The client side of a multi-GPU round in one call per phase:
 * DistributedClient (include/eps/distributed_client.hpp:32-70) over one shard
 * per GPU, each rank also serving the keys k with k % n == rank from `store`
 * (created with shard_id = rank, shard_count = n; every table on every rank).
 * `comm` carries the lookup/push exchanges, `input_comm` (may be NULL: comm)
 * the prepare exchanges, so that a batch can be prepared while the previous
 * round's push runs.  One round of n ranks is what a reference shard serves
 * for one combined request of every rank's features, rank-major.  Every rank
 * must make the same calls in the same order with the same feature schema;
 * input errors are reported on every rank before any data moves. */
typedef struct EpsB200Client EpsB200Client;
EPS_B200_EXPORT int eps_b200_client_create(EpsB200Store* store, EpsB200Comm* comm,
                                           EpsB200Comm* input_comm, EpsB200Client** out,
                                           EpsB200Status* status);
EPS_B200_EXPORT void eps_b200_client_destroy(EpsB200Client* client);
/* PrepareLookupInputs + the key exchange (DistributedClient::LookupPrepared's
 * input), on input_stream; device inputs that stay valid until the lookup.
 * Returns without waiting: it enqueues the partition and the count exchange;
 * the key exchange, which needs the counts on the host, is issued by the next
 * eps_b200_client_prepare (for every earlier batch still pending) or by this
 * batch's lookup, whichever comes first -- the same point on every rank.
 * Preparing two batches ahead therefore never waits on fresh device work.
 * Input errors of any rank are reported by the batch's lookup, on every rank. */
EPS_B200_EXPORT int eps_b200_client_prepare(EpsB200Client* client, const EpsB200Feature* features,
                                            uint64_t count, void* input_stream, uint64_t* prepared,
                                            EpsB200Status* status);
/* Shard lookup + partial exchange + shard-ordered merge of a prepared batch
 * into outputs (device, as eps_b200_lookup's), on `stream`.  Unless read_only,
 * *round receives the handle for eps_b200_client_push. */
EPS_B200_EXPORT int eps_b200_client_lookup(EpsB200Client* client, uint64_t prepared,
                                           EpsB200Buffer* outputs, int32_t read_only, void* stream,
                                           uint64_t* round, EpsB200Status* status);
/* Gradient exchange + one push per shard (DistributedClient::Push).  A
 * non-finite value on any rank rejects the push on every shard; with
 * wait != 0 the rejection is returned here and the round stays pushable or
 * releasable, with wait == 0 it is reported by eps_b200_synchronize. */
EPS_B200_EXPORT int eps_b200_client_push(EpsB200Client* client, uint64_t round,
                                         const EpsB200Buffer* gradients, void* stream, int32_t wait,
                                         EpsB200Status* status);
/* Exchanges of a round, for eps_b200_client_profile. */
enum {
  EPS_B200_EXCHANGE_COUNTS = 0,      /* count rows of a prepared batch */
  EPS_B200_EXCHANGE_KEYS = 1,        /* keys, kept-bag offsets and valid lengths */
  EPS_B200_EXCHANGE_PARTIALS = 2,    /* pooled partials / sequence rows back to the requesters */
  EPS_B200_EXCHANGE_GRADIENTS = 3,   /* gradient rows to the owners */
  EPS_B200_EXCHANGES = 4
};
/* Per-exchange device time (CUDA events around each all-to-all on the stream it
 * is enqueued on, collected when asked), bytes this rank sent to the other
 * ranks, and calls.  No counterpart in the reference (its shards talk over
 * BRPC).  mode 1: reset and start timing, 0: stop, -1: leave as is; bytes and
 * calls are always counted.  Each output (may be NULL) has EPS_B200_EXCHANGES
 * entries. */
EPS_B200_EXPORT int eps_b200_client_profile(EpsB200Client* client, int32_t mode, double* exchange_ms,
                                            uint64_t* exchange_bytes, uint64_t* exchange_calls,
                                            EpsB200Status* status);
/* Drops a prepared batch or an unpushed round (DistributedClient::Release). */
EPS_B200_EXPORT int eps_b200_client_release(EpsB200Client* client, uint64_t handle,
                                            EpsB200Status* status);

/* ---- Agent-style updates with an external optimizer context: the device
 * contract of a GpuCacheAgent (include/eps/cache_backend.hpp:12-29).
 * eps::UpdateContext (include/eps/types.hpp:181-189). */
typedef struct {
  uint32_t table;
  float learning_rate, beta1_power, beta2_power;
  uint64_t optimizer_sequence;
} EpsB200UpdateContext;
/* CacheBackend::ApplyHost (src/cache/host_backend.cpp:119-146): LazyAdam on
 * unique rows of this shard with the context's powers (the table's own powers
 * are not advanced), ++row_updates, all-or-nothing ("cached optimizer
 * overflow").  keys: host; values: [rows][dim] on the host or, with
 * values_on_device, on the store's device.  Waits for the stream. */
EPS_B200_EXPORT int eps_b200_apply_rows(EpsB200Store* store, const EpsB200UpdateContext* context,
                                        const uint64_t* keys, uint64_t rows, const float* values,
                                        int32_t values_on_device, void* stream,
                                        EpsB200Status* status);
/* eps::CompactGradients (include/eps/types.hpp:199-206), host arrays: per target
 * row (keys[rows]) the ordered references row_offsets[rows + 1] into
 * source_rows[refs] / scales[refs] over source_values[sources][dimension]. */
typedef struct {
  const uint64_t* keys; uint64_t rows;
  uint32_t dimension;
  const float* source_values; uint64_t sources;
  const uint64_t* row_offsets;
  const uint64_t* source_rows; const float* scales; uint64_t refs;
} EpsB200CompactGradients;
/* CacheBackend::ApplyCompact (src/cuda/cache_backend.cu:514-539): validation of
 * src/access/compact_gradients.cpp:10-22, the rows expanded on the device in
 * reference order (ExpandCompactGradients, :27-39) and applied as
 * eps_b200_apply_rows. */
EPS_B200_EXPORT int eps_b200_apply_compact(EpsB200Store* store, const EpsB200UpdateContext* context,
                                           const EpsB200CompactGradients* gradients, void* stream,
                                           EpsB200Status* status);

/* ---- Synchronous multi-worker round reduce:
 * SynchronousGradientCollector::Reduce (src/training/synchronous_gradients.cpp:91-126)
 * on the device, for one table of this shard.  Each worker contributes sorted
 * unique keys owned by this shard and float rows [rows][dimension] (device),
 * plus its sample count.  keys_out / values_out (device, capacity >= the sum of
 * the workers' rows) receive the union of the keys in ascending order and
 * float(sum over workers, in worker order, of double(value) * scale) with
 * scale = 1 / denominator: 1 (SUM), the worker count (WORKER_MEAN) or the
 * round's total samples with each worker weighted by its sample count
 * (SAMPLE_MEAN).  *rows receives the number of keys.  The reduced rows are
 * applied like the reference's synchronous applier
 * (src/transport/brpc_synchronous_server.cpp:62-78): one sequence feature of
 * those keys through eps_b200_lookup + eps_b200_push.  Waits for the stream. */
#define EPS_B200_REDUCE_SUM 0
#define EPS_B200_REDUCE_WORKER_MEAN 1
#define EPS_B200_REDUCE_SAMPLE_MEAN 2
typedef struct {
  const uint64_t* keys;     /* device, strictly increasing */
  const float* values;      /* device, [rows][dimension] */
  uint64_t rows;
  uint64_t sample_count;    /* 1 .. 2^40 */
} EpsB200WorkerGradients;
EPS_B200_EXPORT int eps_b200_sync_reduce(EpsB200Store* store, uint32_t table,
                                         const EpsB200WorkerGradients* workers, uint32_t worker_count,
                                         int32_t reduction, uint64_t* keys_out, float* values_out,
                                         uint64_t capacity, uint64_t* rows, void* stream,
                                         EpsB200Status* status);

/* ---- Snapshots in the reference's checksummed shard format (src/store/snapshot.cpp):
 * little-endian, FNV-1a 64 checksum, format 2 (with weight bounds; format 1
 * files are read too).  Write = DrainAndFlush's state file
 * (include/eps/runtime.hpp:116-117): needs no live tickets; holds every row
 * that has been updated (all_rows = 0; a row never updated holds its initial
 * value, which a restore reproduces) or every row of the shard (all_rows = 1);
 * published atomically, never over an existing file.  Read = Restore
 * (include/eps/runtime.hpp:121): new_run must differ from the file's run, the
 * partition (shard, shard count, epoch) and table definitions must match the
 * store's (tables are created first, with their key space); all checks pass
 * before any state changes; then the tables are re-initialised and the file's
 * rows, counters, powers and sequences loaded. */
/* Host-only reading of a snapshot file (no GPU needed; the reference's
 * InspectSnapshot, src/store/snapshot.cpp:190-214, plus the rows): the header,
 * per table its definition, optimizer sequence, powers and row count, and one
 * table's rows (keys, row_updates, [rows][3][dim] = w | m | v).  The checksum
 * and every field are validated as by Restore. */
typedef struct {
  uint32_t format;                 /* 1 or 2 */
  char run[1025];
  uint64_t shard, shard_count, partition_epoch, checksum, tables;
} EpsB200SnapshotInfo;
typedef struct {
  EpsB200Table definition;         /* key_space = 0 (not part of the format) */
  uint64_t optimizer_sequence;
  float beta1_power, beta2_power;
  uint64_t rows;
} EpsB200SnapshotTable;
EPS_B200_EXPORT int eps_b200_snapshot_inspect(const char* path, EpsB200SnapshotInfo* info,
                                              EpsB200SnapshotTable* tables, uint64_t capacity,
                                              EpsB200Status* status);
EPS_B200_EXPORT int eps_b200_snapshot_rows(const char* path, uint64_t table_index, uint64_t* keys,
                                           uint64_t* row_updates, float* state, uint64_t capacity,
                                           EpsB200Status* status);
EPS_B200_EXPORT int eps_b200_snapshot_write(EpsB200Store* store, const char* path, const char* run,
                                            int32_t all_rows, EpsB200Status* status);
EPS_B200_EXPORT int eps_b200_snapshot_read(EpsB200Store* store, const char* path,
                                           const char* new_run, EpsB200Status* status);

/* CpuParameterService::Stats (include/eps/runtime.hpp:134). */
EPS_B200_EXPORT int eps_b200_stats(EpsB200Store* store, EpsB200Stats* stats, EpsB200Status* status);

#ifdef __cplusplus
}
#endif
#endif

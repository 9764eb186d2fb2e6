/* eps_b200_runtime_c.h -- the reference's framework-facing C ABI
 * (include/eps/runtime_c.h of the reference), served by libeps_b200.so so that
 * a consumer that dlopen()s a runtime and calls eps_runtime_api_v1()
 * (adapters/entropy/tensorflow_ops.cc:38-52) can load this library unchanged.
 *
 * The declarations below must be layout-identical to the reference's: field
 * order, types and the function-table order are the contract.  Semantics of
 * the B200 runtime (config keys, supported commands) are described at
 * eps_runtime_api_v1 below. */
#ifndef EPS_B200_RUNTIME_C_H
#define EPS_B200_RUNTIME_C_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define EPS_RUNTIME_ABI 1

/* include/eps/runtime_c.h:9 -- 0 or eps::Error::Code + 1, message copied. */
typedef struct { int32_t code; char message[1024]; } EpsStatus;

/* include/eps/runtime_c.h:10-15 -- host arrays; padding keys are dropped. */
typedef struct {
  uint32_t table, feature, pooling;
  const uint64_t* keys; uint64_t key_count;
  const uint64_t* offsets; uint64_t offset_count;
  int32_t has_padding; uint64_t padding_key;
} EpsFeature;

/* include/eps/runtime_c.h:16-21 -- one feature tensor [rows, columns] f32 on
 * the host (device < 0) or a GPU; owner/release free it, wait(owner, stream)
 * makes `stream` wait until the data is ready. */
typedef struct {
  uint32_t feature; uint64_t rows, columns;
  void* data; int32_t device; void* owner;
  void (*release)(void*);
  int (*wait)(void*, void*, EpsStatus*);
} EpsBuffer;

/* include/eps/runtime_c.h:22 -- the outputs of one pull; handle = lookup
 * ticket for push (UINT64_MAX when a read-only pull was released). */
typedef struct { uint64_t handle, count; EpsBuffer* buffers; void* owner; void (*release)(void*); } EpsBatch;

/* include/eps/runtime_c.h:23 -- a JSON text result. */
typedef struct { const char* data; uint64_t size; void* owner; void (*release)(void*); } EpsText;

/* include/eps/runtime_c.h:24-33 */
typedef struct {
  uint32_t abi_version, struct_bytes;
  int (*create)(const char*, void**, EpsStatus*);
  void (*destroy)(void*);
  int (*pull)(void*, const EpsFeature*, uint64_t, int32_t, int32_t, EpsBatch*, EpsStatus*);
  int (*prepare)(void*, const EpsFeature*, uint64_t, uint64_t*, EpsStatus*);
  int (*pull_prepared)(void*, uint64_t, int32_t, int32_t, EpsBatch*, EpsStatus*);
  int (*push)(void*, uint64_t, const EpsBuffer*, uint64_t, void*, EpsStatus*);
  int (*command)(void*, const char*, const char*, EpsText*, EpsStatus*);
} EpsRuntimeApi;
typedef const EpsRuntimeApi* (*EpsRuntimeEntry)(void);

/* The runtime function table (include/eps/runtime_c.h:40,
 * adapters/entropy/runtime_c.cpp).  B200 runtime:
 *  create(json): {"run": str, "epoch": u64 = 1, "device": int = 0,
 *    "state_bytes": u64, "release_read_only": bool = false,
 *    "snapshot_directory": str = "snapshots",
 *    "tables": [{"id", "dimension", "key_space", "dtype": "float32",
 *      "optimizer": {"kind": "sparse_lazy_adam", "learning_rate", "beta1",
 *        "beta2", "epsilon", "initial_beta1_power", "initial_beta2_power",
 *        "weight_bounds": [min, max]?},
 *      "initialization": {"min", "max", "seed"}}]}
 *    -- one local shard on `device` (the store is the shard; "endpoints" are
 *    ignored); "key_space" is this build's addition (dense tables);
 *    "agents", "cuda" and "training" are rejected (not part of this path).
 *  pull / prepare / pull_prepared: the adapter pull (padding dropped, mean over
 *    the kept keys, sequence positions kept); device != 0 returns GPU buffers
 *    whose wait() makes the consumer's stream wait for the pull.
 *  push: host or device gradients; device gradients are consumed on `stream`
 *    (no copy to the host).
 *  command: "stats", "join", "release" {"handle"}, "cancel_prepared"
 *    {"token"}, "create_table" {table}, "save" {"id"} (a snapshot file per
 *    shard, returned as a JSON array), "endpoint", "close", "abort". */
#if defined(_WIN32)
#define EPS_RUNTIME_EXPORT __declspec(dllexport)
#else
#define EPS_RUNTIME_EXPORT __attribute__((visibility("default")))
#endif
EPS_RUNTIME_EXPORT const EpsRuntimeApi* eps_runtime_api_v1(void);

#ifdef __cplusplus
}
#endif
#endif

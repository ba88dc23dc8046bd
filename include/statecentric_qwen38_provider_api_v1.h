/*
 * Qwen3.8 GDN provider C ABI, version 1 (B200 build).
 *
 * The reference provider includes "statecentric/qwen38_provider_api_v1.h",
 * which is not part of the reference repository.  Every structure and field
 * below is reconstructed from how the provider uses it; the citation beside
 * each declaration names the reference lines that fix its meaning
 * (native/src/qwen38_geometry_normalized_gdn_provider.cpp is abbreviated "P").
 * Field names and order follow that usage.  Numeric enum values are not
 * fixed by the reference and are defined here.
 *
 * Extensions for this build are marked "B200".  They keep the calling
 * convention of the reference: a host loads the library, calls
 * statecentric_qwen38_provider_query_v1() and drives the operator only
 * through the descriptor's function pointers.
 */
#ifndef STATECENTRIC_QWEN38_PROVIDER_API_V1_H_
#define STATECENTRIC_QWEN38_PROVIDER_API_V1_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define STATECENTRIC_QWEN38_PROVIDER_ABI_V1 1u

/* Status codes (P:411-424, 2217-2223, 3570-3637, 3662-3672). */
enum {
  STATECENTRIC_QWEN38_OK = 0,
  STATECENTRIC_QWEN38_INVALID_ARGUMENT = 1,
  STATECENTRIC_QWEN38_INTERNAL = 2,
  STATECENTRIC_QWEN38_TIMEOUT = 3,
  STATECENTRIC_QWEN38_NOT_READY = 4,
  STATECENTRIC_QWEN38_UNSUPPORTED = 5,
  STATECENTRIC_QWEN38_ABI_MISMATCH = 6
};

/* Completion phases (P:3564-3596). */
enum {
  STATECENTRIC_QWEN38_EVENT_PENDING = 0,
  STATECENTRIC_QWEN38_EVENT_COMPLETE = 1
};

/* Tensor scalar types and memory kinds (P:1840-1863). */
enum {
  STATECENTRIC_QWEN38_SCALAR_BF16 = 1,
  STATECENTRIC_QWEN38_SCALAR_F32 = 2
};
enum {
  STATECENTRIC_QWEN38_MEMORY_DEVICE = 1
};

/* Stage and descriptor flags (P:3675-3682). */
#define STATECENTRIC_QWEN38_STAGE_GDN 1u
#define STATECENTRIC_QWEN38_PROVIDER_FLAG_NO_PYTHON_IPC_V1 (1u << 0)

/* Execution flags (P:2259-2303).  The reference admits GDN_FORWARD_V1 alone
 * or together with exactly one of the PREFILL_* variants; all of those start
 * from the hidden state x (inputs x, w_qkv, w_z, w_a, w_b, conv_w, A_log,
 * dt_bias, gamma, w_out; states gdn.conv then gdn.recurrent) and are executed
 * here: projections, causal conv + SiLU and the q/k/v split run on the device
 * before the layer (the PREFILL_* variants only change how the reference
 * splits q/k/v, so all of them run the same kernels).
 * B200: GDN_FORWARD_V1 | GDN_POST_PROJECTION_V6 starts from the projected
 * q, k, v, a, b, z (the reference's precomputed-projection form, P:230-247);
 * GDN_FORWARD_V1 | GDN_OUTPUT_TAIL_V7 runs only the gated-RMSNorm + out_proj
 * tail over o and z (BatchGdnOutputTail, P:1434-1498). */
#define STATECENTRIC_QWEN38_GDN_FORWARD_V1 (1u << 0)
#define STATECENTRIC_QWEN38_GDN_PREFILL_SPLIT_V2 (1u << 1)
#define STATECENTRIC_QWEN38_GDN_PREFILL_SPLIT_V3 (1u << 2)
#define STATECENTRIC_QWEN38_GDN_PREFILL_STRIDED_QKV_V4 (1u << 3)
#define STATECENTRIC_QWEN38_GDN_PREFILL_POST_CONV_PACK_V5 (1u << 4)
#define STATECENTRIC_QWEN38_GDN_POST_PROJECTION_V6 (1u << 5)
#define STATECENTRIC_QWEN38_GDN_OUTPUT_TAIL_V7 (1u << 6)

#define STATECENTRIC_QWEN38_MAX_TENSOR_RANK 8

/* Host services (P:1870-1872, 2434). */
typedef struct statecentric_qwen38_host_v1 {
  uint32_t size;
  uint32_t abi_version;
  void* context;
  uint64_t (*monotonic_time_ns)(void* context);
} statecentric_qwen38_host_v1;

/* Create arguments (P:1869-1881). */
typedef struct statecentric_qwen38_create_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint32_t world_size;
  uint32_t rank;
  int32_t device_ordinal;
  uint32_t assembly_fingerprint_length; /* must be 32 */
  const uint8_t* assembly_fingerprint_sha256;
  const void* configuration;
  uint64_t configuration_length;
} statecentric_qwen38_create_v1;

/* Operator configuration (P:1885-1923).  B200: any head split of the
 * Qwen3-Next / Qwen3.8 GDN geometry is accepted (head_dim 128, value heads a
 * multiple of query heads); max_tokens_per_submission may exceed the
 * reference's 128 (P:256) because long prompts are processed on the device in
 * one submission. */
typedef struct statecentric_qwen38_gdn_create_config_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint32_t hidden_size;
  uint32_t qkv_size_per_rank;
  uint32_t value_size_per_rank;
  uint32_t gate_heads_per_rank;
  uint32_t query_heads_per_rank;
  uint32_t value_heads_per_rank;
  uint32_t head_dim;
  uint32_t max_tokens_per_submission;
  uint32_t prefill_qkv_split_variant;
  uint32_t reserved;
} statecentric_qwen38_gdn_create_config_v1;

/* Tensor view (P:1840-1863).  data is a device address. */
typedef struct statecentric_qwen38_tensor_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint64_t data;
  uint32_t scalar_type;
  uint32_t memory_kind;
  int32_t device_ordinal;
  uint32_t rank;
  uint64_t dimensions[STATECENTRIC_QWEN38_MAX_TENSOR_RANK];
  int64_t strides[STATECENTRIC_QWEN38_MAX_TENSOR_RANK];
  uint64_t byte_length;
} statecentric_qwen38_tensor_v1;

/* Mutable state region (P:2412-2429): state_kind is "gdn.conv" or
 * "gdn.recurrent". */
typedef struct statecentric_qwen38_state_region_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint32_t layer_index;
  uint32_t reserved;
  const char* state_kind;
  statecentric_qwen38_tensor_v1 tensor;
} statecentric_qwen38_state_region_v1;

/* One submission (P:2254-2276, 3163). */
typedef struct statecentric_qwen38_execution_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint32_t rank;
  uint32_t world_size;
  int32_t device_ordinal;
  uint32_t stage;
  uint32_t flags;
  uint32_t layer_index;
  uint64_t token_count;
  uint64_t context_tokens;
  uint64_t stream; /* cudaStream_t of the caller */
  uint32_t input_count;
  uint32_t output_count;
  const statecentric_qwen38_tensor_v1* inputs;
  const statecentric_qwen38_tensor_v1* outputs;
  uint32_t mutable_state_count;
  uint32_t reserved;
  const statecentric_qwen38_state_region_v1* mutable_state;
  uint64_t workspace;        /* host address of gdn_batch_v1 when several states */
  uint64_t workspace_length;
} statecentric_qwen38_execution_v1;

/* Packed multi-sequence metadata, passed through execution.workspace
 * (P:2321-2350).  Offsets must be packed and cover every token. */
typedef struct statecentric_qwen38_gdn_batch_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint64_t state_count;
  uint32_t reserved;
  uint32_t reserved1;
  const uint32_t* token_offsets;
  const uint32_t* token_counts;
} statecentric_qwen38_gdn_batch_v1;

/* Graph-slot binding of the GDN state rows (reference
 * native/include/statecentric/qwen38_gdn_graph_binding.h:15-73, which uses
 * every field below): where the conv and recurrent rows of a batch of at most
 * four sequences live inside a state arena, and whether a captured graph
 * embeds their addresses (DIRECT) or reaches them through private packed
 * buffers that are gathered before and scattered after a replay (COPY).
 * Field order and numeric values are not pinned by the reference. */
#define STATECENTRIC_QWEN38_GDN_BINDING_COPY_V1 1u
#define STATECENTRIC_QWEN38_GDN_BINDING_DIRECT_V1 2u
#define STATECENTRIC_QWEN38_GDN_GRAPH_MAX_ROWS 4
typedef struct statecentric_qwen38_gdn_layout_workspace_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint32_t batch_size;
  uint32_t binding_mode;
  uintptr_t arena;
  uint64_t arena_bytes;
  uint64_t required_arena_bytes;
  uint64_t conv_bytes_per_row;
  uint64_t recurrent_bytes_per_row;
  uintptr_t conv_row_addresses[STATECENTRIC_QWEN38_GDN_GRAPH_MAX_ROWS];
  uintptr_t recurrent_row_addresses[STATECENTRIC_QWEN38_GDN_GRAPH_MAX_ROWS];
} statecentric_qwen38_gdn_layout_workspace_v1;

/* Owned error (P:411-424). */
typedef struct statecentric_qwen38_error_v1 {
  uint32_t size;
  uint32_t abi_version;
  int32_t status;
  uint32_t reserved;
  const char* message;
  void* reserved_pointer;
} statecentric_qwen38_error_v1;

/* Completion record (P:3564-3567). */
typedef struct statecentric_qwen38_completion_v1 {
  uint32_t size;
  uint32_t abi_version;
  uint32_t phase;
  uint32_t reserved;
  uint64_t elapsed_ns;
  uint64_t completed_ns;
} statecentric_qwen38_completion_v1;

typedef struct statecentric_qwen38_provider_handle_v1
    statecentric_qwen38_provider_handle_v1;
typedef struct statecentric_qwen38_event_v1 statecentric_qwen38_event_v1;

/* Descriptor filled by the query entry point (P:3662-3694). */
typedef struct statecentric_qwen38_provider_descriptor_v1 {
  uint32_t size;
  uint32_t abi_version;
  const char* provider_id;      /* "org.statecentric.qwen38.gdn" */
  const char* provider_version; /* "1.0.0" */
  const char* operator_name;    /* "operator.qwen38.gdn" */
  uint32_t operator_version;    /* 1 */
  uint32_t stage;               /* STAGE_GDN */
  uint32_t flags;               /* FLAG_NO_PYTHON_IPC_V1 */
  uint32_t reserved_flags;
  int32_t (*create)(const statecentric_qwen38_host_v1*,
                    const statecentric_qwen38_create_v1*,
                    statecentric_qwen38_provider_handle_v1**,
                    statecentric_qwen38_error_v1**);
  void (*destroy)(statecentric_qwen38_provider_handle_v1*);
  int32_t (*submit)(statecentric_qwen38_provider_handle_v1*,
                    const statecentric_qwen38_execution_v1*,
                    uint64_t deadline_monotonic_ns,
                    statecentric_qwen38_event_v1**,
                    statecentric_qwen38_error_v1**);
  int32_t (*poll)(statecentric_qwen38_provider_handle_v1*,
                  statecentric_qwen38_event_v1*,
                  statecentric_qwen38_completion_v1*,
                  statecentric_qwen38_error_v1**);
  int32_t (*wait)(statecentric_qwen38_provider_handle_v1*,
                  statecentric_qwen38_event_v1*, uint64_t deadline_monotonic_ns,
                  statecentric_qwen38_completion_v1*,
                  statecentric_qwen38_error_v1**);
  int32_t (*cancel)(statecentric_qwen38_provider_handle_v1*,
                    statecentric_qwen38_event_v1*,
                    statecentric_qwen38_error_v1**);
  void (*release_event)(statecentric_qwen38_provider_handle_v1*,
                        statecentric_qwen38_event_v1*);
  void (*release_error)(statecentric_qwen38_error_v1*);
  void* reserved0;
  void* reserved1;
  void* reserved2;
} statecentric_qwen38_provider_descriptor_v1;

#define STATECENTRIC_QWEN38_PROVIDER_DESCRIPTOR_V1_MIN_SIZE \
  offsetof(statecentric_qwen38_provider_descriptor_v1, reserved0)

/* Replaces the reference export of the same name (P:3662-3694). */
#if defined(__GNUC__)
__attribute__((visibility("default")))
#endif
int32_t statecentric_qwen38_provider_query_v1(
    uint32_t host_abi_version, uint32_t host_descriptor_size,
    statecentric_qwen38_provider_descriptor_v1* out_descriptor,
    statecentric_qwen38_error_v1** out_error);

#ifdef __cplusplus
}
#endif

#endif /* STATECENTRIC_QWEN38_PROVIDER_API_V1_H_ */

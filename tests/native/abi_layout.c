/* Prints sizeof/offsetof of the provider ABI structures and the tail group so the test can
 * compare them with the ctypes mirror used by the Python bindings. */
#include <stddef.h>
#include <stdio.h>

#include "gdn_b200.h"
#include "statecentric_qwen38_provider_api_v1.h"

#define F(T, m) printf("%s.%s %zu\n", #T, #m, offsetof(T, m))
#define S(T) printf("%s %zu\n", #T, sizeof(T))

int main(void) {
  S(statecentric_qwen38_host_v1); F(statecentric_qwen38_host_v1, monotonic_time_ns);
  S(statecentric_qwen38_create_v1); F(statecentric_qwen38_create_v1, assembly_fingerprint_sha256);
  F(statecentric_qwen38_create_v1, configuration_length);
  S(statecentric_qwen38_gdn_create_config_v1); F(statecentric_qwen38_gdn_create_config_v1, reserved);
  S(statecentric_qwen38_tensor_v1); F(statecentric_qwen38_tensor_v1, data);
  F(statecentric_qwen38_tensor_v1, dimensions); F(statecentric_qwen38_tensor_v1, strides);
  F(statecentric_qwen38_tensor_v1, byte_length);
  S(statecentric_qwen38_state_region_v1); F(statecentric_qwen38_state_region_v1, tensor);
  S(statecentric_qwen38_execution_v1); F(statecentric_qwen38_execution_v1, stream);
  F(statecentric_qwen38_execution_v1, inputs); F(statecentric_qwen38_execution_v1, mutable_state);
  F(statecentric_qwen38_execution_v1, workspace_length);
  S(statecentric_qwen38_gdn_batch_v1); F(statecentric_qwen38_gdn_batch_v1, token_counts);
  S(statecentric_qwen38_error_v1); F(statecentric_qwen38_error_v1, message);
  S(statecentric_qwen38_completion_v1); F(statecentric_qwen38_completion_v1, completed_ns);
  S(statecentric_qwen38_provider_descriptor_v1);
  F(statecentric_qwen38_provider_descriptor_v1, create);
  F(statecentric_qwen38_provider_descriptor_v1, release_error);
  F(statecentric_qwen38_provider_descriptor_v1, reserved2);
  S(gdn_b200_tail_group_v1); F(gdn_b200_tail_group_v1, max_rows);
  F(gdn_b200_tail_group_v1, hidden); F(gdn_b200_tail_group_v1, region);
  S(statecentric_qwen38_gdn_layout_workspace_v1);
  F(statecentric_qwen38_gdn_layout_workspace_v1, arena);
  F(statecentric_qwen38_gdn_layout_workspace_v1, recurrent_bytes_per_row);
  F(statecentric_qwen38_gdn_layout_workspace_v1, recurrent_row_addresses);
  printf("MIN_SIZE %zu\n", (size_t)STATECENTRIC_QWEN38_PROVIDER_DESCRIPTOR_V1_MIN_SIZE);
  return 0;
}

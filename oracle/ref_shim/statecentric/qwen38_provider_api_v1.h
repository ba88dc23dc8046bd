/* Include shim for compiling the reference's graph-binding header
 * (native/include/statecentric/qwen38_gdn_graph_binding.h) against this
 * repository's reconstruction of the provider ABI header, which the reference
 * includes as "statecentric/qwen38_provider_api_v1.h" but does not ship.
 * Test infrastructure only (oracle/plan_probe.cpp). */
#pragma once
#include "statecentric_qwen38_provider_api_v1.h"

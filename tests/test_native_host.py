"""Host-only native tests (no GPU): compiles and runs the C/C++ truth-table,
buffer-pool and ABI-layout programs under tests/native/ against the library
headers, in the manner of the reference's policy test (distinct exit code per
failing clause)."""
import ctypes
import os
import subprocess

import pytest

import gdn_b200 as G

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "qwen38-gdn-dual-sequence-output-tail_b200", "csrc")
INCLUDE = os.path.join(ROOT, "include")


def _build_and_run(tmp_path, src, cxx=True):
    exe = str(tmp_path / os.path.basename(src).split(".")[0])
    if cxx:
        cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Wpedantic", "-Werror",
               f"-I{CSRC}", f"-I{INCLUDE}", os.path.join(HERE, "native", src), "-o", exe]
    else:
        cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{INCLUDE}",
               os.path.join(HERE, "native", src), "-o", exe]
    subprocess.run(cmd, check=True)
    return subprocess.run([exe], capture_output=True, text=True)


def test_admission_plan_truth_tables(tmp_path):
    r = _build_and_run(tmp_path, "plan_test.cpp")
    assert r.returncode == 0, f"plan truth table failed with code {r.returncode}"


def test_completed_buffer_pool(tmp_path):
    r = _build_and_run(tmp_path, "pool_test.cpp")
    assert r.returncode == 0, f"buffer pool test failed with code {r.returncode}"


def test_provider_abi_layout_matches_python_mirror(tmp_path):
    r = _build_and_run(tmp_path, "abi_layout.c", cxx=False)
    assert r.returncode == 0
    c_layout = dict(line.rsplit(" ", 1) for line in r.stdout.strip().splitlines())
    c_layout = {k: int(v) for k, v in c_layout.items()}
    py = {
        "statecentric_qwen38_host_v1": G.HostV1,
        "statecentric_qwen38_create_v1": G.CreateV1,
        "statecentric_qwen38_gdn_create_config_v1": G.GdnCreateConfigV1,
        "statecentric_qwen38_tensor_v1": G.TensorV1,
        "statecentric_qwen38_state_region_v1": G.StateRegionV1,
        "statecentric_qwen38_execution_v1": G.ExecutionV1,
        "statecentric_qwen38_gdn_batch_v1": G.GdnBatchV1,
        "statecentric_qwen38_error_v1": G.ErrorV1,
        "statecentric_qwen38_completion_v1": G.CompletionV1,
        "statecentric_qwen38_provider_descriptor_v1": G.DescriptorV1,
        "gdn_b200_tail_group_v1": G.TailGroupV1,
        "statecentric_qwen38_gdn_layout_workspace_v1": G.LayoutWorkspaceV1,
    }
    for key, value in c_layout.items():
        if key == "MIN_SIZE":
            assert value == G.DescriptorV1.reserved0.offset
            continue
        if "." in key:
            struct, field = key.split(".")
            assert getattr(py[struct], field).offset == value, key
        else:
            assert ctypes.sizeof(py[key]) == value, key


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", G.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    import re
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    declared = set()
    for header in ("gdn_b200.h", "statecentric_qwen38_provider_api_v1.h"):
        text = open(os.path.join(INCLUDE, header)).read()
        declared |= set(re.findall(r"GDN_B200_API\s+[\w\s\*]+?\b(gdn_b200_\w+)\s*\(", text))
        declared |= set(re.findall(r"\b(statecentric_qwen38_provider_query_v1)\s*\(", text))
    assert set(G.EXPORTED_SYMBOLS) <= declared
    assert declared <= exported, declared - exported
    for name in declared:
        getattr(G.lib(), name)


def test_graph_binding_rules(tmp_path):
    r = _build_and_run(tmp_path, "graph_binding_test.cpp")
    assert r.returncode == 0, f"graph binding test failed with code {r.returncode}"


def test_plans_and_graph_binding_match_the_reference_headers(tmp_path):
    """Bit-exact agreement with the reference's own admission and binding code.

    ``oracle/plan_probe.cpp`` is compiled against the reference's headers
    where they lie (qwen38_gdn_dual_sequence_tail_policy.h,
    qwen38_gdn_geometry_policy.h and qwen38_gdn_graph_binding.h, the last one
    against this repository's reconstructed provider ABI header, which must
    therefore provide every field it reads) into ``oracle/_ref/``, and against
    ``gdn_plan.h`` / ``gdn_graph_binding.h``.  Both print every feature
    predicate over all flag combinations, the chunk-vs-recurrent rule, every
    plan over all gates x token-count vectors of length 0-4 (admitted cases
    listed, every answer hashed) and 20000 COPY-binding cases (refusal message
    or the full copy sequence); the outputs must be identical."""
    oracle = os.path.join(ROOT, "oracle")
    ref_bin = os.path.join(oracle, "_ref", "plan_probe_ref")
    if os.path.isdir("/root/reference/native/include"):
        subprocess.run(["make", "-s", "-C", oracle, "ref"], check=True)
    if not os.path.exists(ref_bin):
        pytest.skip("the reference headers are not present and oracle/_ref was not built")
    repo_bin = str(tmp_path / "plan_probe_repo")
    subprocess.run(["make", "-s", "-C", oracle, "probe", f"PROBE_OUT={repo_bin}"], check=True)
    ref = subprocess.run([ref_bin], capture_output=True, text=True, check=True).stdout
    ours = subprocess.run([repo_bin], capture_output=True, text=True, check=True).stdout
    assert ref.count("\n") > 20000
    assert "admitted=8" in ref
    ref_lines, our_lines = ref.splitlines(), ours.splitlines()
    assert len(ref_lines) == len(our_lines)
    diff = [(a, b) for a, b in zip(ref_lines, our_lines) if a != b]
    assert not diff, diff[:5]

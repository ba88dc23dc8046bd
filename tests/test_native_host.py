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

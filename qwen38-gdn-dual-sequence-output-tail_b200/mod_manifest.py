"""Engine manifest and activation contract for the B200 GDN provider.

The reference ships its provider to the engine as a frozen, SHA-256-bound
candidate: an immutable directory holding the provider library and its
contracts, described by a mod manifest (``versions/<v>/mod.json``:
``schema_version``, ``mod_id``, ``target``, ``activation`` with the
environment and the artifacts bound by ``sha256``) and an activation
contract written by its freezing script
(``scripts/freeze_qwen38_tp2pp2_gdn_dual_sequence_tail_activation.sh``:
schema, revision, the bound hashes, the activation chain,
``performance_claim``).  This module does the same for this build:

    python mod_manifest.py freeze <candidate_dir> --revision r001 [--world-size N]
    python mod_manifest.py verify <candidate_dir>

``freeze`` refuses an existing directory, copies ``libgdn_b200.so`` and the
ABI headers into it, reads the provider descriptor from the copied library
(``statecentric_qwen38_provider_query_v1``; no GPU needed), writes the
activation contract and the manifest with every artifact bound by SHA-256,
and makes the files read-only.  ``verify`` re-hashes every bound artifact and
re-queries the library, and raises on any difference.
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import json
import os
import shutil
import stat
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_NAME = "libgdn_b200.so"
HEADERS = ("gdn_b200.h", "statecentric_qwen38_provider_api_v1.h")
MANIFEST_SCHEMA = "statecentric-native-mod-v1"
ACTIVATION_SCHEMA = "statecentric-qwen38-gdn-b200-activation-v1"
MOD_ID = "qwen38.gdn-b200-layer-hot-path"
PROVIDER_ENV = "STATECENTRIC_QWEN38_GDN_PROVIDER_LIBRARY"


class ManifestError(RuntimeError):
    pass


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _descriptor(lib_path: str) -> dict:
    """The provider descriptor of the library at lib_path."""
    sys.path.insert(0, HERE)
    import gdn_b200 as G
    lib = ctypes.CDLL(lib_path)
    fn = lib.statecentric_qwen38_provider_query_v1
    fn.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(G.DescriptorV1), G._ErrPP]
    fn.restype = ctypes.c_int32
    d = G.DescriptorV1()
    err = ctypes.POINTER(G.ErrorV1)()
    st = fn(G.ABI_V1, ctypes.sizeof(G.DescriptorV1), ctypes.byref(d), ctypes.byref(err))
    if st != G.OK:
        raise ManifestError(f"provider query failed with status {st}")
    return {"abi_version": int(d.abi_version), "provider_id": d.provider_id.decode(),
            "provider_version": d.provider_version.decode(),
            "operator_name": d.operator_name.decode(), "operator_version": int(d.operator_version),
            "stage": int(d.stage), "flags": int(d.flags)}


def freeze(candidate_dir: str, revision: str, world_size: int = 1,
           lib_path: str | None = None) -> dict:
    """Writes an immutable candidate directory; returns the manifest."""
    lib_path = lib_path or os.path.join(HERE, LIB_NAME)
    if os.path.exists(candidate_dir):
        raise ManifestError(f"refusing to overwrite candidate: {candidate_dir}")
    if not os.path.exists(lib_path):
        raise ManifestError(f"provider library missing: {lib_path}")
    if world_size not in (1, 2, 4, 8):
        raise ManifestError("world_size must be 1, 2, 4 or 8")
    os.makedirs(candidate_dir)
    shutil.copy2(lib_path, os.path.join(candidate_dir, LIB_NAME))
    for h in HEADERS:
        shutil.copy2(os.path.join(ROOT, "include", h), os.path.join(candidate_dir, h))
    provider = os.path.join(candidate_dir, LIB_NAME)
    descriptor = _descriptor(provider)
    provider_sha = sha256(provider)
    activation = {
        "schema": ACTIVATION_SCHEMA,
        "revision": revision,
        "provider_sha256": provider_sha,
        "descriptor": descriptor,
        "execution_flags": {
            "GDN_FORWARD_V1": "the layer from the hidden state x (input projections, causal "
                              "conv, chunked or recurrent core, flattened output tail)",
            "GDN_FORWARD_V1|GDN_POST_PROJECTION_V6": "the layer from projected q, k, v, a, b, z",
            "GDN_FORWARD_V1|GDN_OUTPUT_TAIL_V7": "the gated RMSNorm + out_proj tail only",
        },
        "activation_chain": [
            f"engine exports {PROVIDER_ENV}=<candidate>/{LIB_NAME}",
            "engine dlopens the library and calls statecentric_qwen38_provider_query_v1",
            f"engine checks abi_version {descriptor['abi_version']} and provider_id "
            f"{descriptor['provider_id']}",
            "engine creates one provider per rank (world_size, rank, device_ordinal) and routes "
            "the GDN stage's submissions to it",
        ],
        "performance_claim": False,
    }
    act_path = os.path.join(candidate_dir, "gdn-b200-activation.json")
    with open(act_path, "w") as f:
        json.dump(activation, f, indent=2, sort_keys=True)
    artifacts = [{"role": "gdn-provider", "uri": LIB_NAME, "sha256": provider_sha},
                 {"role": "activation-contract", "uri": os.path.basename(act_path),
                  "sha256": sha256(act_path)}]
    artifacts += [{"role": "abi-header", "uri": h, "sha256": sha256(os.path.join(candidate_dir, h))}
                  for h in HEADERS]
    manifest = {
        "schema_version": MANIFEST_SCHEMA,
        "mod_id": MOD_ID,
        "version": revision,
        "title": "B200 GDN layer hot path (chunked prefill, recurrent decode, flattened tail)",
        "summary": "sm_100a kernels behind the Qwen3.8 GDN provider C ABI.",
        "status": "candidate",
        "default_enabled": False,
        "target": {
            "model": {"family": "Qwen3-Next / Qwen3.8 gated delta net layer"},
            "topology": {"world_size": world_size, "tensor_parallel_size": world_size},
            "accelerator": {"vendor": "NVIDIA", "device": "B200", "arch": "sm_100a",
                            "device_count": world_size},
        },
        "activation": {
            "mode": "environment-and-artifact-binding",
            "status": "manual-engine-route",
            "environment": {PROVIDER_ENV: LIB_NAME},
            "artifacts": artifacts,
        },
    }
    with open(os.path.join(candidate_dir, "mod.json"), "w") as f:
        json.dump(manifest, f, indent=2, sort_keys=True)
    for name in os.listdir(candidate_dir):
        p = os.path.join(candidate_dir, name)
        os.chmod(p, stat.S_IRUSR | stat.S_IRGRP | stat.S_IROTH |
                 (stat.S_IXUSR if name.endswith(".so") else 0))
    return manifest


def verify(candidate_dir: str) -> dict:
    """Re-checks every SHA-256 binding and the provider descriptor."""
    with open(os.path.join(candidate_dir, "mod.json")) as f:
        manifest = json.load(f)
    if manifest.get("schema_version") != MANIFEST_SCHEMA or manifest.get("mod_id") != MOD_ID:
        raise ManifestError("not a manifest of this provider")
    by_role = {}
    for a in manifest["activation"]["artifacts"]:
        path = os.path.join(candidate_dir, a["uri"])
        if not os.path.isfile(path) or sha256(path) != a["sha256"]:
            raise ManifestError(f"binding failed: {a['uri']}")
        by_role.setdefault(a["role"], a)
    with open(os.path.join(candidate_dir, by_role["activation-contract"]["uri"])) as f:
        activation = json.load(f)
    if activation.get("schema") != ACTIVATION_SCHEMA:
        raise ManifestError("activation contract schema")
    if activation["provider_sha256"] != by_role["gdn-provider"]["sha256"]:
        raise ManifestError("activation contract names another provider")
    if _descriptor(os.path.join(candidate_dir, LIB_NAME)) != activation["descriptor"]:
        raise ManifestError("provider descriptor differs from the activation contract")
    return manifest


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    f = sub.add_parser("freeze")
    f.add_argument("candidate_dir")
    f.add_argument("--revision", required=True)
    f.add_argument("--world-size", type=int, default=1)
    v = sub.add_parser("verify")
    v.add_argument("candidate_dir")
    args = ap.parse_args(argv)
    try:
        if args.cmd == "freeze":
            freeze(args.candidate_dir, args.revision, args.world_size)
        verify(args.candidate_dir)
    except ManifestError as e:
        print(f"{args.cmd} failed: {e}", file=sys.stderr)
        return 3
    print(f"{args.cmd} ok: {args.candidate_dir}")
    return 0


if __name__ == "__main__":
    sys.exit(main())

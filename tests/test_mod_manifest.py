"""Engine manifest and activation contract of the provider (the freezing and
SHA-256 binding the reference does for its candidates,
scripts/freeze_qwen38_tp2pp2_gdn_dual_sequence_tail_activation.sh and
versions/0.1.2/mod.json): freeze a candidate, verify it, and refuse a
tampered artifact or an existing directory.  CPU only."""
import json
import os
import stat

import pytest

import mod_manifest as M


def test_freeze_then_verify(tmp_path):
    cand = str(tmp_path / "cand")
    manifest = M.freeze(cand, "r001", world_size=8)
    assert manifest["target"]["accelerator"]["arch"] == "sm_100a"
    assert manifest["target"]["topology"]["world_size"] == 8
    roles = {a["role"] for a in manifest["activation"]["artifacts"]}
    assert {"gdn-provider", "activation-contract", "abi-header"} <= roles
    assert M.verify(cand) == manifest
    act = json.load(open(os.path.join(cand, "gdn-b200-activation.json")))
    assert act["descriptor"]["provider_id"] == "org.statecentric.qwen38.gdn"
    assert act["descriptor"]["operator_name"] == "operator.qwen38.gdn"
    assert act["performance_claim"] is False
    # frozen: read-only files
    assert not os.stat(os.path.join(cand, "mod.json")).st_mode & stat.S_IWUSR


def test_refuses_existing_candidate(tmp_path):
    cand = str(tmp_path / "cand")
    os.makedirs(cand)
    with pytest.raises(M.ManifestError, match="refusing to overwrite"):
        M.freeze(cand, "r001")


def test_tampered_artifact_fails_binding(tmp_path):
    cand = str(tmp_path / "cand")
    M.freeze(cand, "r001")
    hdr = os.path.join(cand, "gdn_b200.h")
    os.chmod(hdr, 0o644)
    with open(hdr, "a") as f:
        f.write("\n/* edited */\n")
    with pytest.raises(M.ManifestError, match="binding failed: gdn_b200.h"):
        M.verify(cand)


def test_cli(tmp_path):
    cand = str(tmp_path / "c2")
    assert M.main(["freeze", cand, "--revision", "r002", "--world-size", "2"]) == 0
    assert M.main(["verify", cand]) == 0
    assert M.main(["freeze", cand, "--revision", "r002"]) == 3

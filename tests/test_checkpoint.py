"""Checkpoints in the reference's format (crates/staleynet-model/src/checkpoint.rs): byte layout, manifest field
names, optimizer-state order, load_weights' rules (copied / grown by rows / fresh / mismatch). CPU only."""
import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from staleynet_b200 import checkpoint as ck  # noqa: E402


def test_layout_is_the_references(tmp_path):
    """tensors.bin: little-endian f32, parameters in manifest order, then every first moment, then every second
    moment (checkpoint.rs:1-3, 263-271); model.json uses the serde names of CheckpointMetadata and TensorEntry."""
    params = {"a": torch.arange(3, dtype=torch.float32), "b": torch.arange(2, dtype=torch.float32) + 10}
    first = {"a": torch.full((3,), 0.5), "b": torch.full((2,), 0.25)}
    second = {"a": torch.full((3,), 2.0), "b": torch.full((2,), 4.0)}
    ck.save(tmp_path, params, {"width": 8}, step=7, training={"lr": 1e-3}, first_moments=first, second_moments=second)
    raw = np.fromfile(tmp_path / "tensors.bin", dtype="<f4")
    assert raw.tolist() == [0, 1, 2, 10, 11, 0.5, 0.5, 0.5, 0.25, 0.25, 2, 2, 2, 4, 4]
    meta = json.loads((tmp_path / "model.json").read_text())
    assert set(meta) == {"model", "tensors", "step", "has_optimizer_state", "training"}
    assert meta["tensors"] == [{"name": "a", "len": 3}, {"name": "b", "len": 2}]
    assert meta["step"] == 7 and meta["has_optimizer_state"] is True
    assert not (tmp_path / "tensors.bin.partial").exists()
    got = ck.read(tmp_path, device="cpu")
    assert torch.equal(got.parameters["b"], params["b"])
    assert torch.equal(got.first_moments["a"], first["a"]) and torch.equal(got.second_moments["b"], second["b"])


def test_load_weights_copies_grows_by_rows_and_keeps_fresh(tmp_path):
    ck.save(tmp_path, {"pos": torch.ones(2, 4), "w": torch.full((3, 3), 2.0)}, {}, step=0)
    model = {"pos": torch.zeros(3, 4), "w": torch.zeros(3, 3), "new": torch.full((2,), 5.0)}
    t = ck.load_weights(tmp_path, model)
    assert t.copied == ["w"] and t.grown == ["pos"] and t.fresh == ["new"]
    assert model["pos"][:2].eq(1).all() and model["pos"][2].eq(0).all() and model["w"].eq(2).all()
    with pytest.raises(ValueError, match="values in the checkpoint"):
        ck.load_weights(tmp_path, {"w": torch.zeros(2, 5)})


def test_truncated_file_is_refused(tmp_path):
    ck.save(tmp_path, {"a": torch.zeros(4)}, {}, step=0)
    raw = np.fromfile(tmp_path / "tensors.bin", dtype="<f4")
    raw[:2].tofile(tmp_path / "tensors.bin")
    with pytest.raises(ValueError, match="ends before"):
        ck.read(tmp_path, device="cpu")


@pytest.mark.gpu
def test_read_uploads_into_one_device_buffer(tmp_path):
    params = {f"t{i}": torch.randn(1000 + i) for i in range(5)}
    ck.save(tmp_path, params, {}, step=1)
    got = ck.read(tmp_path, device="cuda")
    for k, v in params.items():
        assert got.parameters[k].is_cuda and torch.equal(got.parameters[k].cpu(), v)
    assert got.parameters["t1"].data_ptr() == got.parameters["t0"].data_ptr() + 4 * 1000

"""Checkpoints in the reference's format (crates/staleynet-model/src/checkpoint.rs:1-171): a directory holding
`model.json` — {"model": <ModelConfig>, "tensors": [{"name", "len"}, ...], "step", "has_optimizer_state",
"training"} — and `tensors.bin`, little-endian f32 values: every parameter in manifest order, then (when
has_optimizer_state) every AdamW first moment followed by every second moment, in the same order.

Reading maps `tensors.bin` and moves it to the GPU in one pinned host-to-device copy; parameters are then slices of
that device buffer (`read`), or copied into existing device tensors by name (`load_weights`, the reference's rules:
a stored tensor smaller than the parameter by whole rows fills its leading rows — a grown position table — and any
other size mismatch is an error). Writing (`save`) uses the reference's `.partial` file and rename, so a reader never
sees a half-written file.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

METADATA_FILE = "model.json"
TENSOR_FILE = "tensors.bin"


@dataclass
class Checkpoint:
    """A checkpoint read into device memory: `parameters` and (when stored) `first_moments` / `second_moments` map
    tensor names to 1-D f32 views of one device buffer, in manifest order."""

    metadata: dict
    parameters: dict
    first_moments: dict = field(default_factory=dict)
    second_moments: dict = field(default_factory=dict)


@dataclass
class WeightTransfer:
    """What `load_weights` did (checkpoint.rs:81-93)."""

    copied: list = field(default_factory=list)
    grown: list = field(default_factory=list)
    fresh: list = field(default_factory=list)


def read_metadata(directory) -> dict:
    return json.loads((Path(directory) / METADATA_FILE).read_text())


def _values(directory) -> np.ndarray:
    return np.fromfile(Path(directory) / TENSOR_FILE, dtype="<f4")


def _upload(values: np.ndarray, device):
    """One pinned host-to-device copy of the whole file."""
    import torch

    host = torch.from_numpy(values.astype(np.float32, copy=False))
    if device is None or torch.device(device).type == "cpu":
        return host
    staged = torch.empty(host.numel(), dtype=torch.float32, pin_memory=True)
    staged.copy_(host)
    out = torch.empty(host.numel(), dtype=torch.float32, device=device)
    out.copy_(staged, non_blocking=True)
    torch.cuda.current_stream(out.device).synchronize()
    return out


def read(directory, device="cuda") -> Checkpoint:
    """Reads a checkpoint into one device buffer (`load`, checkpoint.rs:137-165, without building the model)."""
    metadata = read_metadata(directory)
    entries = metadata["tensors"]
    values = _values(directory)
    count = sum(int(e["len"]) for e in entries)
    expected = count * (3 if metadata.get("has_optimizer_state") else 1)
    if values.size < expected:
        raise ValueError(f"tensors.bin ends before every tensor was read ({values.size} of {expected} values)")
    buffer = _upload(values[:expected], device)
    parameters, firsts, seconds = {}, {}, {}
    offset = 0
    for e in entries:
        parameters[e["name"]] = buffer[offset:offset + int(e["len"])]
        offset += int(e["len"])
    if metadata.get("has_optimizer_state"):
        for target in (firsts, seconds):
            for e in entries:
                target[e["name"]] = buffer[offset:offset + int(e["len"])]
                offset += int(e["len"])
    return Checkpoint(metadata, parameters, firsts, seconds)


def load_weights(directory, model_parameters: dict, row_widths: dict | None = None) -> WeightTransfer:
    """Copies stored tensors into `model_parameters` (name -> device tensor) by name (checkpoint.rs:95-134): equal
    sizes are copied whole; a stored tensor shorter than the parameter by whole rows (`row_widths[name]` values per
    row, else the parameter's last dimension) fills the leading rows; parameters the checkpoint lacks stay as they
    are. Any other size mismatch raises ValueError."""
    ckpt = read(directory, device=next(iter(model_parameters.values())).device if model_parameters else "cuda")
    transfer = WeightTransfer()
    for name, param in model_parameters.items():
        source = ckpt.parameters.get(name)
        if source is None:
            transfer.fresh.append(name)
            continue
        width = (row_widths or {}).get(name, param.shape[-1] if param.dim() > 0 else 1)
        grows = source.numel() < param.numel() and source.numel() % width == 0
        if source.numel() != param.numel() and not grows:
            raise ValueError(f"{name} has {source.numel()} values in the checkpoint but {param.numel()} in the model")
        param.view(-1)[:source.numel()].copy_(source)
        (transfer.grown if grows else transfer.copied).append(name)
    return transfer


def _write_atomically(path: Path, write) -> None:
    staging = path.with_name(path.name + ".partial")
    with open(staging, "wb") as f:
        write(f)
        f.flush()
    os.replace(staging, path)


def save(directory, parameters: dict, model_config: dict, step: int, training=None, first_moments: dict | None = None,
         second_moments: dict | None = None) -> None:
    """Writes `parameters` (name -> tensor, in the model's visitor order) and optionally the AdamW moments in the
    reference's layout (checkpoint.rs:42-78)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    names = list(parameters)
    has_opt = first_moments is not None and second_moments is not None

    def host(t):
        return t.detach().float().reshape(-1).cpu().numpy().astype("<f4", copy=False)

    def write(f):
        for n in names:
            host(parameters[n]).tofile(f)
        if has_opt:
            for n in names:
                host(first_moments[n]).tofile(f)
            for n in names:
                host(second_moments[n]).tofile(f)

    _write_atomically(directory / TENSOR_FILE, write)
    metadata = {"model": model_config, "tensors": [{"name": n, "len": int(parameters[n].numel())} for n in names],
                "step": int(step), "has_optimizer_state": has_opt, "training": training}
    _write_atomically(directory / METADATA_FILE, lambda f: f.write(json.dumps(metadata, indent=2).encode()))

"""Host side of the on-device checkpoint restore: the safetensors header is read
exactly as the safetensors library writes it (the reference's on-disk format,
formats/safetensors.py:1-15), and the loader refuses host destinations."""

from __future__ import annotations

import json
import os

import pytest
import torch
from safetensors.torch import load_file, save_file

from llada_quant_b200 import checkpoint as C


def _write(tmp_path):
    g = torch.Generator().manual_seed(0)
    state = {
        "blocks.0._qw1": torch.randint(-128, 127, (4, 64, 32), generator=g, dtype=torch.int8),
        "blocks.0._sw1": torch.rand(4, 64, 1, generator=g),
        "blocks.0._qw2": torch.randint(-128, 127, (4, 32, 16), generator=g, dtype=torch.int8),
        "blocks.0._sw2": torch.rand(4, 32, 1, generator=g),
        "embed.weight": torch.randn(10, 8, generator=g).to(torch.bfloat16),
        "norm.bias": torch.zeros(3, dtype=torch.float16),
    }
    path = os.path.join(tmp_path, "model-int4.safetensors")
    save_file(state, path)
    with open(os.path.join(tmp_path, "quantization.json"), "w") as f:
        json.dump({"config": {"bits": 4, "compute_dtype": "bfloat16"},
                   "targets": [{"kind": "expert", "name": "blocks.0"}]}, f)
    return state, path


def test_header_matches_the_safetensors_library(tmp_path):
    state, path = _write(str(tmp_path))
    header, start = C.read_header(path)
    assert set(header) == set(state)
    ref = load_file(path)
    raw = open(path, "rb").read()
    for name, e in header.items():
        assert list(ref[name].shape) == e["shape"]
        assert C._DTYPES[e["dtype"]] == ref[name].dtype
        lo, hi = e["data_offsets"]
        got = torch.frombuffer(bytearray(raw[start + lo:start + hi]), dtype=ref[name].dtype).reshape(ref[name].shape)
        assert torch.equal(got, ref[name])


def test_find_weights_file_and_host_refusal(tmp_path):
    _, path = _write(str(tmp_path))
    assert C.find_weights_file(str(tmp_path)) == path
    with pytest.raises(FileNotFoundError):
        C.find_weights_file(str(tmp_path / "nowhere"))
    with pytest.raises(RuntimeError, match="GPU"):
        C.load_to_device(path, "cpu")
    assert C.read_manifest(str(tmp_path))["config"]["bits"] == 4

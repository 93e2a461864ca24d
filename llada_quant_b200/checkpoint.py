"""Quantized checkpoints restored straight into GPU memory (formats/safetensors.py:103-167).

The reference loads the whole ``model-int*.safetensors`` file into host tensors
(``load_file(..., device="cpu")``), copies them into the model with
``load_state_dict`` and then rebuilds the PACKED access
(``restore_llada_experts_from_buffers``, adapters/llada_moe.py:163-186).  Here the
file is parsed directly: its header gives every tensor's dtype, shape and byte
range, the bytes are read through two pinned staging buffers and copied into
their final device tensors with asynchronous host-to-device copies (a read of
the next chunk overlaps the copy of the previous one), and the packed expert
buffers come out as ready :class:`PackedExperts` handles -- the kernels' input
contract -- with no host copy of the model and no second device copy.
The on-disk format is the reference's, unchanged.
"""

from __future__ import annotations

import glob
import json
import os
import struct
from typing import Dict, Iterable, Optional, Tuple

import torch
import torch.nn as nn

from .moe import PACKED_BUFFERS, PackedExperts, QuantExpertWeights, attach_packed_buffers
from .moe import install_packed_expert_access, is_packed_expert_block, quant_result_from_buffers

WEIGHTS_GLOB = "model-int*.safetensors"
MANIFEST_FILENAME = "quantization.json"

_DTYPES = {
    "BOOL": torch.bool, "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16, "I32": torch.int32,
    "I64": torch.int64, "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32,
    "F64": torch.float64,
}


def find_weights_file(directory: str) -> str:
    """formats/safetensors.py:86-92."""
    matches = sorted(glob.glob(os.path.join(directory, WEIGHTS_GLOB)))
    if not matches:
        raise FileNotFoundError(f"no {WEIGHTS_GLOB} in {directory!r}")
    if len(matches) > 1:
        raise RuntimeError(f"ambiguous checkpoint, multiple weight files: {matches}")
    return matches[0]


def read_header(path: str) -> Tuple[Dict[str, dict], int]:
    """The safetensors header: ``{name: {dtype, shape, data_offsets}}`` and where the data starts."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path!r} is not a safetensors file")
        (n,) = struct.unpack("<Q", raw)
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    for name, entry in header.items():
        if entry["dtype"] not in _DTYPES:
            raise ValueError(f"{name}: unsupported safetensors dtype {entry['dtype']}")
    return header, 8 + n


def load_to_device(path: str, device, names: Optional[Iterable[str]] = None,
                   chunk_bytes: int = 64 << 20) -> Dict[str, torch.Tensor]:
    """Every tensor of the file (or ``names``) as a tensor on ``device``, read in file order
    through two pinned staging buffers of ``chunk_bytes``."""
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("load_to_device restores into GPU memory only")
    header, data_start = read_header(path)
    wanted = set(header) if names is None else set(names)
    missing = wanted - set(header)
    if missing:
        raise KeyError(f"not in {path!r}: {sorted(missing)}")
    entries = sorted(((header[n]["data_offsets"][0], header[n]["data_offsets"][1], n) for n in wanted))
    out: Dict[str, torch.Tensor] = {}
    dst_bytes: Dict[str, torch.Tensor] = {}
    for _, _, n in entries:
        e = header[n]
        t = torch.empty(e["shape"], dtype=_DTYPES[e["dtype"]], device=device)
        out[n] = t
        dst_bytes[n] = t.view(-1).view(torch.uint8) if t.numel() else t
    stream = torch.cuda.Stream(device)
    # the destinations come from the caching allocator on the current stream: a block
    # freed there may still be read by queued kernels, so the copies start after them
    stream.wait_stream(torch.cuda.current_stream(device))
    stage = [torch.empty(chunk_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    done = [None, None]
    with open(path, "rb", buffering=0) as f, torch.cuda.stream(stream):
        k = 0
        for lo, hi, n in entries:
            pos = lo
            while pos < hi:
                span = min(hi - pos, chunk_bytes)
                buf = stage[k & 1]
                if done[k & 1] is not None:
                    done[k & 1].synchronize()  # the copy that last used this buffer has finished
                f.seek(data_start + pos)
                view = memoryview(buf.numpy())[:span]
                got = f.readinto(view)
                if got != span:
                    raise IOError(f"short read in {path!r} at {data_start + pos}")
                dst_bytes[n][pos - lo:pos - lo + span].copy_(buf[:span], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
                done[k & 1] = ev
                pos += span
                k += 1
    stream.synchronize()
    return out


def read_manifest(directory: str) -> dict:
    path = os.path.join(directory, MANIFEST_FILENAME)
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        return json.load(f)


def load_packed_experts(source: str, device, bits: Optional[int] = None) -> Dict[str, PackedExperts]:
    """Every fused expert block of a checkpoint (directory or weights file) as a
    :class:`PackedExperts` on ``device``, keyed by module name.  ``bits`` defaults to
    the manifest's ``config.bits``; the group size is derived from each scale tensor
    (runtime/moe.py:82-102)."""
    path = find_weights_file(source) if os.path.isdir(source) else source
    if bits is None:
        cfg = read_manifest(os.path.dirname(path)).get("config") or {}
        bits = cfg.get("bits")
        if bits is None:
            raise ValueError("bits not given and no quantization.json config beside the weights")
    header, _ = read_header(path)
    prefixes = sorted({n[: -len(b)] for n in header for b in PACKED_BUFFERS if n.endswith(b)})
    names = [p + b for p in prefixes for b in PACKED_BUFFERS]
    absent = [n for n in names if n not in header]
    if absent:
        raise RuntimeError(f"incomplete packed expert buffers in {path!r}: {absent}")
    state = load_to_device(path, device, names)
    blocks: Dict[str, PackedExperts] = {}
    for p in prefixes:
        q1, s1, q2, s2 = (state[p + b] for b in PACKED_BUFFERS)
        group = quant_result_from_buffers(q1, s1, bits).group_size
        blocks[p.rstrip(".")] = PackedExperts(q1, s1, q2, s2, bits, group)
    return blocks


def restore_quantized_weights(model: nn.Module, directory: str, device=None, strict: bool = True) -> dict:
    """``load_quantized_weights`` (formats/safetensors.py:138-167) for PACKED models, restored
    straight into ``device`` (default: the model's first parameter or buffer device).
    Missing buffers are registered on the fly; the BF16 expert weights are expected to be
    absent.  Returns the manifest dict."""
    manifest = read_manifest(directory)
    cfg = manifest.get("config") or {}
    if device is None:
        ref = next(iter(list(model.parameters()) + list(model.buffers())), None)
        device = ref.device if ref is not None and ref.is_cuda else torch.device("cuda")
    state = load_to_device(find_weights_file(directory), device)
    existing = dict(model.state_dict())
    expected_missing = set()
    for t in manifest.get("targets", []):
        if t.get("kind") == "expert":
            prefix = f"{t['name']}." if t.get("name") else ""
            expected_missing.update({prefix + "w1", prefix + "w2"})
    unexpected = []
    for name, tensor in state.items():
        parent, _, leaf = name.rpartition(".")
        try:
            module = model.get_submodule(parent) if parent else model
        except AttributeError as exc:
            raise RuntimeError(
                f"state dict mismatch: checkpoint holds {name!r} but the model has no submodule "
                f"{parent!r} ({exc}). The checkpoint was produced from a different architecture.") from exc
        if name in existing:
            with torch.no_grad():
                cur = existing[name]
                if isinstance(cur, nn.Parameter) or leaf in module._parameters:
                    module._parameters[leaf] = nn.Parameter(tensor, requires_grad=cur.requires_grad)
                else:
                    module._buffers[leaf] = tensor
        elif leaf.startswith("_"):
            module.register_buffer(leaf, tensor, persistent=True)
        else:
            unexpected.append(name)
    missing = [k for k in existing if k not in state and k not in expected_missing]
    if strict and (missing or unexpected):
        raise RuntimeError(f"state dict mismatch: missing={missing}, unexpected={unexpected}")
    bits = cfg.get("bits")
    if bits is not None:
        compute_dtype = getattr(torch, cfg.get("compute_dtype", "bfloat16"))
        for block in model.modules():
            if not all(hasattr(block, b) for b in PACKED_BUFFERS):
                continue
            weights = QuantExpertWeights(w1=quant_result_from_buffers(block._qw1, block._sw1, bits),
                                         w2=quant_result_from_buffers(block._qw2, block._sw2, bits))
            attach_packed_buffers(block, weights, compute_dtype, cfg.get("compile_dequant", False))
            if not is_packed_expert_block(block):
                install_packed_expert_access(block)
    return manifest

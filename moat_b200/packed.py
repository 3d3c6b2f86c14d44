"""On-disk INT4 super-block weights: a safetensors file of 144-byte streams.

Each weight is stored as one ``uint8[nsb * 144]`` tensor (the reference's
``struct SuperBlock`` wire form, ``antigravity-engine/src/shaders/batched_gemm.metal:17-20``)
and described in the file's ``__metadata__`` by a JSON record: its original shape,
element count before padding, quantizer variant (``engine``: divide by the fp16 scale,
``quantize_weights_int4``; ``toplevel``: divide by the fp32 scale,
``quantize_fp16_to_int4``) and group size. The loader mirrors the reference's
``ModelWeightLoader`` (``antigravity-engine/src/model_loader.py:34-133``): quantize and
repack a layer, pad its flat weights to a multiple of 256 with zeros, keep a memory
budget, dequantize a layer back to its original shape.
"""

from __future__ import annotations

import json
from typing import Dict, Optional

import numpy as np

FORMAT = "moat-int4-superblock-144"
SUPERBLOCK_BYTES = 144
SUPERBLOCK_ELEMS = 256


def _record(shape, n_elements: int, variant: str, group_size: int = 32) -> str:
    return json.dumps({"format": FORMAT, "shape": [int(s) for s in shape], "n_elements": int(n_elements),
                       "variant": variant, "group_size": int(group_size)})


def save_packed(path: str, layers: Dict[str, dict]) -> None:
    """Write ``{name: {"superblocks": uint8 stream, "original_shape": shape,
    "n_elements": n, "variant": "engine"|"toplevel"}}`` as one safetensors file."""
    from safetensors.numpy import save_file
    tensors, meta = {}, {"format": FORMAT}
    for name, layer in layers.items():
        sb = layer["superblocks"]
        if hasattr(sb, "detach"):  # torch tensor (any device)
            sb = sb.detach().cpu().numpy()
        sb = np.ascontiguousarray(np.asarray(sb, dtype=np.uint8).reshape(-1))
        if sb.size % SUPERBLOCK_BYTES != 0:
            raise ValueError(f"{name}: stream of {sb.size} bytes is not whole super-blocks")
        n = int(layer.get("n_elements", sb.size // SUPERBLOCK_BYTES * SUPERBLOCK_ELEMS))
        if not 0 < n <= sb.size // SUPERBLOCK_BYTES * SUPERBLOCK_ELEMS:
            raise ValueError(f"{name}: n_elements {n} does not fit {sb.size // SUPERBLOCK_BYTES} super-blocks")
        tensors[name] = sb
        meta[name] = _record(layer.get("original_shape", (n,)), n, layer.get("variant", "engine"),
                             layer.get("group_size", 32))
    save_file(tensors, path, metadata=meta)


def load_packed(path: str, device: Optional[str] = None) -> Dict[str, dict]:
    """Read a file written by :func:`save_packed`. ``device`` (e.g. ``"cuda:0"``) puts
    each stream on that GPU as a torch uint8 tensor; otherwise NumPy arrays."""
    from safetensors import safe_open
    out = {}
    with safe_open(path, framework="numpy") as f:
        meta = f.metadata() or {}
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path} is not a {FORMAT} file")
        for name in f.keys():
            rec = json.loads(meta[name])
            sb = f.get_tensor(name)
            if sb.dtype != np.uint8 or sb.ndim != 1 or sb.size % SUPERBLOCK_BYTES != 0:
                raise ValueError(f"{name}: not a super-block stream")
            if device is not None:
                from . import _lib
                t = _lib.torch()
                sb = t.from_numpy(np.ascontiguousarray(sb)).to(device)
            out[name] = {"superblocks": sb, "original_shape": tuple(rec["shape"]), "n_elements": rec["n_elements"],
                         "variant": rec["variant"], "group_size": rec["group_size"],
                         "memory_bytes": int(sb.numel() if hasattr(sb, "numel") else sb.size)}
    return out


class PackedWeightLoader:
    """GPU counterpart of the reference's ``ModelWeightLoader``
    (``model_loader.py:34-133``): layers are quantized and packed on the device, kept
    as 144-byte streams, and saved to / loaded from one safetensors file."""

    def __init__(self, memory_budget_bytes: int = int(2.5 * 1024 ** 3), device: str = "cuda:0"):
        self.memory_budget_bytes = memory_budget_bytes
        self.device = device
        self.layers: Dict[str, dict] = {}
        self.total_loaded_bytes = 0

    def load_and_repack_layer(self, layer_name: str, weights_fp16, group_size: int = 32,
                              variant: str = "engine") -> dict:
        """Quantize (``variant`` semantics) and pack one weight; flat weights are
        padded with zeros to a multiple of 256 as in model_loader.py:66-72."""
        if group_size != 32:
            raise ValueError("the super-block format has group size 32")
        from . import _lib
        from .dequant import quantize_to_superblocks
        t = _lib.torch()
        shape = tuple(weights_fp16.shape)
        w = weights_fp16 if isinstance(weights_fp16, t.Tensor) else t.from_numpy(
            np.ascontiguousarray(np.asarray(weights_fp16, dtype=np.float16)))
        w = w.to(self.device).reshape(-1).to(t.float16)
        n = w.numel()
        pad = (-n) % SUPERBLOCK_ELEMS
        if pad:
            w = t.cat([w, t.zeros(pad, dtype=w.dtype, device=w.device)])
        nbytes = (n + pad) // SUPERBLOCK_ELEMS * SUPERBLOCK_BYTES
        if self.total_loaded_bytes + nbytes > self.memory_budget_bytes:
            raise MemoryError(
                f"Loading layer '{layer_name}' ({nbytes / 1e6:.1f} MB) exceeds memory budget of "
                f"{self.memory_budget_bytes / 1e9:.2f} GB. Currently loaded: {self.total_loaded_bytes / 1e9:.2f} GB.")
        sb = quantize_to_superblocks(w, variant=variant)
        layer = {"layer_name": layer_name, "original_shape": shape, "n_elements": n, "superblocks": sb,
                 "memory_bytes": nbytes, "variant": variant, "group_size": group_size}
        self.layers[layer_name] = layer
        self.total_loaded_bytes += nbytes
        return layer

    def dequantize_layer(self, layer_name: str):
        """fp16 weights of a loaded layer in its original shape (padding trimmed)."""
        if layer_name not in self.layers:
            raise KeyError(f"Layer '{layer_name}' not found in loader")
        from .dequant import unpack_superblock_weights
        layer = self.layers[layer_name]
        sb = layer["superblocks"]
        n_sb = (sb.numel() if hasattr(sb, "numel") else sb.size) // SUPERBLOCK_BYTES
        flat = unpack_superblock_weights(sb, n_sb)
        return flat.reshape(-1)[:layer["n_elements"]].reshape(layer["original_shape"])

    def save(self, path: str) -> None:
        save_packed(path, self.layers)

    def load(self, path: str) -> None:
        """Add every layer of a packed file (streams go to this loader's device)."""
        for name, layer in load_packed(path, device=self.device).items():
            if self.total_loaded_bytes + layer["memory_bytes"] > self.memory_budget_bytes:
                raise MemoryError(f"Loading layer '{name}' exceeds memory budget")
            layer["layer_name"] = name
            self.layers[name] = layer
            self.total_loaded_bytes += layer["memory_bytes"]


__all__ = ["FORMAT", "save_packed", "load_packed", "PackedWeightLoader"]

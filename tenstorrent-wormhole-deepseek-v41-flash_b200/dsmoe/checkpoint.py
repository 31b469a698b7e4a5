"""Checkpoint loader: DeepSeek-V4.1-Flash safetensors shards -> resident expert store.

Replaces the reference's checkpoint path for the MoE layers: the raw-bytes safetensors reader
(dsv41/ckpt.py:18-50), the per-expert projection decode (ckpt.py:41-50) and the host packing into
Tenstorrent tiles cached on disk (dsv41/tt/store.py:66-89). Here the checkpoint's bytes go to the
GPU as they are and dsmoe_store_pack_expert repacks them there once (this rank's tensor-parallel
slice only); nothing is dequantized on the host.

Tensor formats read (the ones the reference handles, ckpt.py:3-6 and dsv41/tt/weights.py:45-61):
  routed experts   layers.L.ffn.experts.E.w{1,2,3}.weight  I8 [out, in/2], two e2m1 codes per byte,
                   low nibble first;  .scale  F8_E8M0 [out, in/32]  -> the FP4 store as they are
  shared expert    layers.L.ffn.shared_experts.w{1,2,3}.weight  F8_E4M3 [out, in];  .scale
                   F8_E8M0 [ceil(out/128), ceil(in/128)]  -> the FP8 store, scale 2^(byte-127) in fp32
                   (exact)
  router           layers.L.ffn.gate.weight  (F32 or BF16) [E, H];  .bias  F32 [E];  .bias_vl optional
"""
import json
import mmap
import os
import struct
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from .synth import ExpertWeights, RouterWeights

_NP = {"F32": np.float32, "BF16": np.uint16, "I8": np.uint8, "U8": np.uint8, "F8_E4M3": np.uint8,
       "F8_E8M0": np.uint8, "F16": np.float16, "I64": np.int64}


class SafetensorsCheckpoint:
    """Zero-copy reader of a sharded safetensors checkpoint (``model.safetensors.index.json`` plus
    shards, or a single ``.safetensors`` file): each shard is mapped once and tensors are returned as
    numpy views of their bytes."""

    def __init__(self, path: str):
        if os.path.isdir(path):
            with open(os.path.join(path, "model.safetensors.index.json")) as f:
                wm = json.load(f)["weight_map"]
            self.files = {name: os.path.join(path, fn) for name, fn in wm.items()}
        else:
            self.files = None
            self._single = path
        self._shards: Dict[str, Tuple[mmap.mmap, int, dict]] = {}

    def _shard(self, fn: str):
        s = self._shards.get(fn)
        if s is None:
            with open(fn, "rb") as f:
                n = struct.unpack("<Q", f.read(8))[0]
                hdr = json.loads(f.read(n))
                hdr.pop("__metadata__", None)
                mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
            s = self._shards[fn] = (mm, 8 + n, hdr)
        return s

    def _file_of(self, name: str) -> str:
        if self.files is None:
            return self._single
        if name not in self.files:
            raise KeyError(name)
        return self.files[name]

    def has(self, name: str) -> bool:
        try:
            return name in self._shard(self._file_of(name))[2]
        except KeyError:
            return False

    def raw(self, name: str):
        """(numpy view of the tensor in its storage type, safetensors dtype string, shape)."""
        mm, base, hdr = self._shard(self._file_of(name))
        meta = hdr[name]
        a, b = meta["data_offsets"]
        dt = meta["dtype"]
        if dt not in _NP:
            raise ValueError(f"{name}: unsupported dtype {dt}")
        t = np.frombuffer(mm, dtype=_NP[dt], count=(b - a) // np.dtype(_NP[dt]).itemsize, offset=base + a)
        return t.reshape(meta["shape"]), dt, list(meta["shape"])

    def tensor(self, name: str) -> torch.Tensor:
        """A CPU torch tensor of the raw storage (uint8 for the 8-bit and packed formats)."""
        t, dt, _ = self.raw(name)
        out = torch.from_numpy(np.array(t))  # copy out of the mapping
        return out.view(torch.bfloat16) if dt == "BF16" else out

    def close(self):
        for mm, _, _ in self._shards.values():
            mm.close()
        self._shards.clear()


def _e8m0_to_f32(b: torch.Tensor) -> torch.Tensor:
    """E8M0 bytes -> 2^(b - 127) in fp32, exactly (0xFF -> NaN as in the format)."""
    e = b.to(torch.int32)
    out = torch.ldexp(torch.ones_like(e, dtype=torch.float32), e - 127)
    return torch.where(e == 255, torch.full_like(out, float("nan")), out)


def routed_expert(ck: SafetensorsCheckpoint, layer: int, e: int, prefix: str = "layers") -> ExpertWeights:
    """One MXFP4 routed expert as checkpoint bytes (ckpt.py:41-50 reads the same tensors)."""
    stem = f"{prefix}.{layer}.ffn.experts.{e}"
    parts = []
    for pj in ("w1", "w3", "w2"):
        q, qd, qs = ck.raw(f"{stem}.{pj}.weight")
        s, sd, ss = ck.raw(f"{stem}.{pj}.scale")
        if qd not in ("I8", "U8") or sd != "F8_E8M0":
            raise ValueError(f"{stem}.{pj}: expected packed e2m1 + e8m0, got {qd} + {sd}")
        if ss != [qs[0], qs[1] * 2 // 32]:
            raise ValueError(f"{stem}.{pj}: scale shape {ss} does not match {qs}")
        parts += [torch.from_numpy(np.array(q)), torch.from_numpy(np.array(s))]
    w1, s1, w3, s3, w2, s2 = parts
    return ExpertWeights("fp4", w1, s1, w3, s3, w2, s2)


def shared_expert(ck: SafetensorsCheckpoint, layer: int, prefix: str = "layers") -> ExpertWeights:
    """The shared expert: e4m3 weights with e8m0 128 x 128 block scales -> FP8 store input."""
    stem = f"{prefix}.{layer}.ffn.shared_experts"
    parts = []
    for pj in ("w1", "w3", "w2"):
        q, qd, qs = ck.raw(f"{stem}.{pj}.weight")
        s, sd, ss = ck.raw(f"{stem}.{pj}.scale")
        if qd != "F8_E4M3" or sd != "F8_E8M0":
            raise ValueError(f"{stem}.{pj}: expected e4m3 + e8m0 block scales, got {qd} + {sd}")
        if ss != [-(-qs[0] // 128), -(-qs[1] // 128)]:
            raise ValueError(f"{stem}.{pj}: scale shape {ss} is not 128 x 128 blocks of {qs}")
        parts += [torch.from_numpy(np.array(q)), _e8m0_to_f32(torch.from_numpy(np.array(s)))]
    w1, s1, w3, s3, w2, s2 = parts
    return ExpertWeights("fp8", w1, s1, w3, s3, w2, s2)


def router(ck: SafetensorsCheckpoint, layer: int, prefix: str = "layers") -> RouterWeights:
    f = f"{prefix}.{layer}.ffn.gate"
    wg = ck.tensor(f"{f}.weight").float()
    bias = ck.tensor(f"{f}.bias").float()
    bias_vl = ck.tensor(f"{f}.bias_vl").float() if ck.has(f"{f}.bias_vl") else None
    return RouterWeights(wg, bias, bias_vl)


def load_layer(moe, ck: SafetensorsCheckpoint, layer: int, prefix: str = "layers",
               experts: Optional[range] = None) -> None:
    """Fill ``moe`` (a dsmoe.MoE of fmt "fp4") from the checkpoint's layer ``layer``: router, shared
    expert, every routed expert (or ``experts``). Each expert's bytes go to the GPU once and are
    repacked there into this rank's slice of the resident store."""
    if moe.fmt != "fp4":
        raise ValueError("the checkpoint's routed experts are MXFP4: build the layer with fmt='fp4'")
    moe.load_router(router(ck, layer, prefix))
    moe.load_shared(shared_expert(ck, layer, prefix))
    for e in (experts if experts is not None else range(moe.n_experts)):
        moe.load_expert(e, routed_expert(ck, layer, e, prefix))


def write_safetensors(path: str, tensors: Dict[str, Tuple[np.ndarray, str]]) -> None:
    """A minimal safetensors writer (``{name: (array, dtype string)}``), for tests and tooling."""
    hdr, blobs, off = {}, [], 0
    for name, (arr, dt) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        hdr[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(hdr).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)

"""Checkpoint / resume of a TrainableTransformer and its Adam state.

forge-llm itself only exports weights (`exportWeights`, train.js:199-220,
fed to exportGGUF); resuming a run also needs Adam's m, v and step counter
(autograd.js:214-220).  One file holds all of it:

    8 bytes   magic b"FORGECK1"
    4 bytes   header length n (little-endian uint32)
    n bytes   JSON header: format version, model config, parameter count,
              Adam hyper-parameters and step, and for every section its byte
              offset (from the end of the header), length and CRC-32
    sections  little-endian float32 arrays in the flat parameter order of
              the model: "params", then "adam_m", "adam_v" when saved

The file is written to a temporary name and renamed into place, so a crash
mid-write leaves the previous checkpoint intact.  Loading checks the magic,
the header, the configuration, the sizes and every CRC before it touches the
model, and restores the device-side Adam step counter as well, so a step
captured as a CUDA graph resumes on the same schedule.
"""
from __future__ import annotations

import json
import os
import struct
import zlib

import numpy as np

MAGIC = b"FORGECK1"
VERSION = 1
_ADAM_KEYS = ("lr", "b1", "b2", "eps", "wd", "clip", "total")


def write_file(path: str, header: dict, sections: dict) -> None:
    """Write `sections` (name -> float32 array) with `header` to `path`
    atomically."""
    index, off = [], 0
    for name, arr in sections.items():
        a = np.ascontiguousarray(arr, dtype="<f4").ravel()
        sections[name] = a
        index.append({"name": name, "offset": off, "bytes": a.nbytes, "crc32": zlib.crc32(a.data) & 0xFFFFFFFF})
        off += a.nbytes
    h = dict(header, format=VERSION, sections=index)
    hb = json.dumps(h, sort_keys=True).encode()
    tmp = f"{path}.tmp.{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<I", len(hb)))
        f.write(hb)
        for a in sections.values():
            f.write(a.data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def read_file(path: str) -> tuple[dict, dict]:
    """(header, name -> float32 array) of a checkpoint file; ValueError if it
    is not one, is truncated, or a section fails its CRC."""
    with open(path, "rb") as f:
        blob = f.read()
    if len(blob) < 12 or blob[:8] != MAGIC:
        raise ValueError(f"{path}: not a forgellm checkpoint")
    (n,) = struct.unpack("<I", blob[8:12])
    if 12 + n > len(blob):
        raise ValueError(f"{path}: truncated header")
    try:
        header = json.loads(blob[12:12 + n])
    except ValueError as e:
        raise ValueError(f"{path}: unreadable header ({e})") from None
    if header.get("format") != VERSION:
        raise ValueError(f"{path}: checkpoint format {header.get('format')} (this build reads {VERSION})")
    base, out = 12 + n, {}
    for s in header["sections"]:
        lo, hi = base + s["offset"], base + s["offset"] + s["bytes"]
        if hi > len(blob) or s["bytes"] % 4:
            raise ValueError(f"{path}: section {s['name']} truncated")
        raw = blob[lo:hi]
        if zlib.crc32(raw) & 0xFFFFFFFF != s["crc32"]:
            raise ValueError(f"{path}: section {s['name']} fails its CRC-32")
        out[s["name"]] = np.frombuffer(raw, dtype="<f4").copy()
    return header, out


def _config_dict(cfg) -> dict:
    return {k: (float(v) if isinstance(v, float) else v) for k, v in vars(cfg).items()
            if isinstance(v, (int, float, str, bool))}


def save_checkpoint(path: str, model, opt=None, extra: dict | None = None) -> None:
    """Parameters (and, with `opt`, Adam's m, v and step) of `model`."""
    import torch
    torch.cuda.synchronize()
    header = {"config": _config_dict(model.cfg), "n_params": model.countParams(), "extra": extra or {}}
    sections = {"params": model.flat_params.detach().cpu().numpy()}
    if opt is not None:
        if getattr(opt, "m_flat", None) is None:
            raise ValueError("save_checkpoint: the optimizer must hold the model's flat parameters")
        header["adam"] = dict({k: getattr(opt, k) for k in _ADAM_KEYS}, t=int(opt.t))
        sections["adam_m"] = opt.m_flat.detach().cpu().numpy()
        sections["adam_v"] = opt.v_flat.detach().cpu().numpy()
    write_file(path, header, sections)


def load_checkpoint(path: str, model, opt=None) -> dict:
    """Restore what save_checkpoint wrote into `model` (and `opt`).  Returns
    the header.  Nothing is modified unless every check passes."""
    import torch
    header, sec = read_file(path)
    want = _config_dict(model.cfg)
    if header["config"] != want:
        diff = sorted(k for k in set(want) | set(header["config"]) if want.get(k) != header["config"].get(k))
        raise ValueError(f"{path}: model configuration differs ({', '.join(diff)})")
    n = model.countParams()
    if header["n_params"] != n or sec["params"].size != n:
        raise ValueError(f"{path}: {sec['params'].size} parameters, the model has {n}")
    if opt is not None:
        if "adam" not in header:
            raise ValueError(f"{path}: no optimizer state was saved")
        if getattr(opt, "m_flat", None) is None:
            raise ValueError("load_checkpoint: the optimizer must hold the model's flat parameters")
        if sec["adam_m"].size != n or sec["adam_v"].size != n:
            raise ValueError(f"{path}: optimizer state has the wrong size")
    dev = model.flat_params.device
    with torch.no_grad():
        model.flat_params.copy_(torch.from_numpy(sec["params"]).to(dev))
        if opt is not None:
            opt.m_flat.copy_(torch.from_numpy(sec["adam_m"]).to(dev))
            opt.v_flat.copy_(torch.from_numpy(sec["adam_v"]).to(dev))
            for k in _ADAM_KEYS:
                setattr(opt, k, header["adam"][k])
            opt.t = int(header["adam"]["t"])
            if getattr(opt, "_t_dev", None) is not None:
                opt._t_dev.fill_(opt.t)
    model._shadow_stale = True
    if getattr(model, "flat_params_bf16", None) is not None:
        # the bf16 weight copy the fused GEMMs read is rebuilt now: a step
        # replayed from a CUDA graph runs no host code that would refresh it
        model.bf16_weights()
    torch.cuda.synchronize()
    return header

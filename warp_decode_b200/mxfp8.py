"""MXFP8 weight packing: quantise once, at load time, on the device.

Format (OCP Microscaling Formats v1.0, MXFP8 with E4M3 elements):
blocks of 32 consecutive weights along the reduction axis (the last axis of
both ``w_gate_up [E, 2I, H]`` and ``w_down [E, H, I]``) share one E8M0 scale.
The shared exponent is ``floor(log2(max|w|)) - 8`` (8 = exponent of the
largest E4M3 normal, 448), elements are ``w / 2^exp`` rounded to nearest-even
E4M3 and saturated at +-448, and the scale byte stores ``exp + 127``.
An all-zero block gets the smallest scale (byte 0).

The kernels consume ``q`` (uint8 bit patterns, same shape as the weights) and
``scale`` (uint8, last axis / 32) directly (the MXFP8 entry points of the C
ABI).  ``save_mxfp8`` / ``load_mxfp8`` persist packed weights in a versioned
file, and ``load_or_quantize_moe`` is the quantise-once loader of one MoE
layer's weights.
"""
from __future__ import annotations

import torch

BLOCK = 32
E4M3_MAX = 448.0


def quantize_mxfp8(w: torch.Tensor, chunk_rows: int = 4096):
    """Quantise along the last axis.  Returns (q uint8, scale uint8)."""
    if w.shape[-1] % BLOCK:
        raise ValueError("last axis must be a multiple of 32")
    shape = w.shape
    flat = w.reshape(-1, shape[-1])
    q = torch.empty(flat.shape, dtype=torch.uint8, device=w.device)
    s = torch.empty(flat.shape[0], shape[-1] // BLOCK, dtype=torch.uint8, device=w.device)
    for r0 in range(0, flat.shape[0], chunk_rows):
        blk = flat[r0:r0 + chunk_rows].float().reshape(-1, shape[-1] // BLOCK, BLOCK)
        amax = blk.abs().amax(dim=-1)
        # floor(log2(amax)) exactly: amax = m * 2^ex with m in [0.5, 1)
        _, ex = torch.frexp(amax)
        e = torch.where(amax > 0, ex.to(torch.int32) - 1 - 8, torch.full_like(ex, -127, dtype=torch.int32))
        e = e.clamp(-127, 127)
        scaled = torch.ldexp(blk, (-e).to(torch.float32)[..., None])
        scaled = scaled.clamp(-E4M3_MAX, E4M3_MAX)
        q[r0:r0 + chunk_rows] = scaled.to(torch.float8_e4m3fn).view(torch.uint8).reshape(-1, shape[-1])
        s[r0:r0 + chunk_rows] = (e + 127).to(torch.uint8)
    return q.reshape(shape), s.reshape(*shape[:-1], shape[-1] // BLOCK)


def dequantize_mxfp8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """float32 weights: e4m3(q) * 2^(scale - 127) per block of 32."""
    vals = q.view(torch.float8_e4m3fn).float()
    shape = vals.shape
    blk = vals.reshape(*shape[:-1], shape[-1] // BLOCK, BLOCK)
    out = torch.ldexp(blk, (scale.to(torch.float32) - 127.0)[..., None])
    return out.reshape(shape)


# ---------------------------------------------------------------------------
# Persisted format: quantise once, load many times
# ---------------------------------------------------------------------------
# A packed-weight file holds named (q, scale) pairs:
#
#   bytes 0..3    magic b"WDMX"
#   bytes 4..7    format version (little-endian uint32, FILE_VERSION)
#   bytes 8..11   header length L (little-endian uint32)
#   bytes 12..    L bytes of UTF-8 JSON:
#                 {"format": "mxfp8-e4m3-ue8m0", "block": 32, "axis": -1,
#                  "meta": {...caller's...},
#                  "tensors": {name: {"shape": [...], "scale_shape": [...],
#                                     "q": [offset, nbytes, sha256],
#                                     "scale": [offset, nbytes, sha256]}}}
#   payload       raw uint8 arrays at 256-byte aligned offsets, counted from
#                 the first 256-byte boundary after the header (the kernels'
#                 layouts: q [..., K] row-major, scale [..., K/32] row-major,
#                 K = the reduction axis)
#
# The loader rejects a file whose magic, version, format, block size, shapes,
# sizes or checksums do not match, instead of handing wrong bytes to a kernel.
FILE_MAGIC = b"WDMX"
FILE_VERSION = 1
FILE_FORMAT = "mxfp8-e4m3-ue8m0"
_ALIGN = 256


def _sha256(buf) -> str:
    import hashlib

    return hashlib.sha256(buf).hexdigest()


def save_mxfp8(path, tensors: dict, meta: dict | None = None) -> None:
    """Write named (q, scale) pairs (uint8 tensors, any device) to `path`."""
    import json
    import struct

    entries, blobs, off = {}, [], 0
    for name, (q, s) in tensors.items():
        q = q.detach().to("cpu").contiguous()
        s = s.detach().to("cpu").contiguous()
        if q.dtype != torch.uint8 or s.dtype != torch.uint8:
            raise ValueError(f"{name}: q and scale must be uint8")
        if q.shape[-1] % BLOCK or tuple(s.shape) != tuple(q.shape[:-1]) + (q.shape[-1] // BLOCK,):
            raise ValueError(f"{name}: scale shape {tuple(s.shape)} does not match q {tuple(q.shape)}")
        rec = {"shape": list(q.shape), "scale_shape": list(s.shape)}
        for key, t in (("q", q), ("scale", s)):
            b = t.numpy().tobytes()
            rec[key] = [off, len(b), _sha256(b)]
            blobs.append((off, b))
            off += (len(b) + _ALIGN - 1) // _ALIGN * _ALIGN
        entries[name] = rec
    header = json.dumps({"format": FILE_FORMAT, "block": BLOCK, "axis": -1, "meta": meta or {},
                         "tensors": entries}, sort_keys=True).encode()
    base = (12 + len(header) + _ALIGN - 1) // _ALIGN * _ALIGN
    with open(path, "wb") as f:
        f.write(FILE_MAGIC + struct.pack("<II", FILE_VERSION, len(header)) + header)
        f.write(b"\0" * (base - 12 - len(header)))
        pos = 0
        for o, b in blobs:
            f.write(b"\0" * (o - pos))
            f.write(b)
            pos = o + len(b)


def load_mxfp8(path, device=None, verify: bool = True):
    """Read a file written by save_mxfp8: returns ({name: (q, scale)}, meta).

    Raises ValueError for a file that is not a packed-weight file of this
    version and format, or whose sizes or checksums do not match."""
    import json
    import struct

    import numpy as np

    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 12 or data[:4] != FILE_MAGIC:
        raise ValueError(f"{path}: not an MXFP8 packed-weight file (bad magic)")
    version, hlen = struct.unpack("<II", data[4:12])
    if version != FILE_VERSION:
        raise ValueError(f"{path}: format version {version}, this loader reads {FILE_VERSION}")
    if 12 + hlen > len(data):
        raise ValueError(f"{path}: truncated header")
    try:
        hdr = json.loads(data[12:12 + hlen].decode())
    except Exception as e:
        raise ValueError(f"{path}: unreadable header ({e})") from None
    if hdr.get("format") != FILE_FORMAT or hdr.get("block") != BLOCK or hdr.get("axis") != -1:
        raise ValueError(f"{path}: format {hdr.get('format')!r} block {hdr.get('block')!r} "
                         f"axis {hdr.get('axis')!r}, expected {FILE_FORMAT!r} block {BLOCK} axis -1")
    base = (12 + hlen + _ALIGN - 1) // _ALIGN * _ALIGN
    out = {}
    for name, rec in hdr["tensors"].items():
        shape, sshape = tuple(rec["shape"]), tuple(rec["scale_shape"])
        if not shape or shape[-1] % BLOCK or sshape != shape[:-1] + (shape[-1] // BLOCK,):
            raise ValueError(f"{path}: {name}: inconsistent shapes {shape} / {sshape}")
        arrs = []
        for key, shp in (("q", shape), ("scale", sshape)):
            off, nbytes, digest = rec[key]
            if nbytes != int(np.prod(shp)) or base + off + nbytes > len(data):
                raise ValueError(f"{path}: {name}.{key}: size does not match the shape or the file")
            b = data[base + off: base + off + nbytes]
            if verify and _sha256(b) != digest:
                raise ValueError(f"{path}: {name}.{key}: checksum mismatch")
            t = torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).reshape(shp)
            arrs.append(t.to(device) if device is not None else t)
        out[name] = tuple(arrs)
    return out, hdr.get("meta", {})


def load_or_quantize_moe(path, w_gate_up: torch.Tensor | None = None,
                         w_down: torch.Tensor | None = None, device=None):
    """The quantise-once loader of an MoE layer's MXFP8 weights.

    If `path` exists it is loaded (and checked against the bf16 weights'
    shapes when they are given); otherwise w_gate_up [E, 2I, H] and w_down
    [E, H, I] are quantised (on their device) and written to `path`.
    Returns (gate_up_q, gate_up_scale, down_q, down_scale) on `device`
    (default: the weights' device, else the CPU)."""
    import os

    if device is None and w_gate_up is not None:
        device = w_gate_up.device
    if os.path.exists(path):
        t, meta = load_mxfp8(path, device=device)
        if set(t) != {"w_gate_up", "w_down"}:
            raise ValueError(f"{path}: expected tensors w_gate_up and w_down, found {sorted(t)}")
        for name, w in (("w_gate_up", w_gate_up), ("w_down", w_down)):
            if w is not None and tuple(t[name][0].shape) != tuple(w.shape):
                raise ValueError(f"{path}: {name} has shape {tuple(t[name][0].shape)}, the model "
                                 f"{tuple(w.shape)}")
        (gq, gs), (dq, ds) = t["w_gate_up"], t["w_down"]
        return gq, gs, dq, ds
    if w_gate_up is None or w_down is None:
        raise FileNotFoundError(f"{path} does not exist and no weights were given to quantise")
    E, two_i, H = w_gate_up.shape
    if tuple(w_down.shape) != (E, H, two_i // 2):
        raise ValueError(f"w_down shape {tuple(w_down.shape)} does not match w_gate_up "
                         f"{tuple(w_gate_up.shape)}")
    gq, gs = quantize_mxfp8(w_gate_up)
    dq, ds = quantize_mxfp8(w_down)
    save_mxfp8(path, {"w_gate_up": (gq, gs), "w_down": (dq, ds)},
               meta={"experts": E, "hidden": H, "inter": two_i // 2})
    if device is not None:
        gq, gs, dq, ds = (t.to(device) for t in (gq, gs, dq, ds))
    return gq, gs, dq, ds

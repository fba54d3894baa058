"""On-disk form of the tile-first FP8 weights, so that `relayout` becomes a load instead of a permute.

The reference re-packs every eligible weight on each start-up (patches/fp8_hand_sm89.py:652-672: the
row-major e4m3 [N, K] weight is permuted to tiles[nb][kb][r][c] = W[nb*128 + r][kb*128 + c] on the GPU,
H:667). This module stores that packed form, with its block scales, once; later starts read the bytes
straight into the tile buffers the GEMM kernels consume.

File layout (all integers little-endian):

    offset 0   8 bytes   magic b"BSFP8TL1"
    offset 8   8 bytes   header length H
    offset 16  H bytes   UTF-8 JSON header
    ...        zero padding to the next multiple of 4096
    blobs      each starts at a multiple of 4096 (offsets in the header are absolute)

Header:

    {"format": "bsfp8-tiles", "version": 1, "block": 128,
     "layout": "tiles[nb][kb][r][c] = W[nb*128 + r][kb*128 + c]",
     "entries": {name: {"N": N, "K": K,
                        "tiles": {"offset": o, "nbytes": N*K, "sha256": hex},
                        "scale": {"offset": o, "nbytes": 4*(N/128)*(K/128), "sha256": hex}}}}

`tiles` are the e4m3 bytes in tile-first order ([N/128, K/128, 128, 128]); `scale` is the fp32
weight_scale_inv [N/128, K/128], row-major. The digests cover the stored bytes; `load(verify=True)`
checks them.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from pathlib import Path

import torch

MAGIC = b"BSFP8TL1"
FORMAT = "bsfp8-tiles"
VERSION = 1
BLOCK = 128
ALIGN = 4096
LAYOUT = "tiles[nb][kb][r][c] = W[nb*128 + r][kb*128 + c]"


class TilePackError(ValueError):
    """A tile-pack file that is malformed or does not match the weights it is loaded for."""


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def _bytes_of(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()


def _check_entry(name: str, tiles: torch.Tensor, scale: torch.Tensor) -> tuple[int, int]:
    if tiles.dim() != 4 or tiles.shape[2:] != (BLOCK, BLOCK) or tiles.element_size() != 1:
        raise TilePackError(f"{name}: tiles must be 1-byte [N/128, K/128, 128, 128], got {tuple(tiles.shape)} "
                            f"{tiles.dtype}")
    N, K = tiles.shape[0] * BLOCK, tiles.shape[1] * BLOCK
    if scale.dtype != torch.float32 or tuple(scale.shape) != (N // BLOCK, K // BLOCK):
        raise TilePackError(f"{name}: scale must be fp32 [{N // BLOCK}, {K // BLOCK}], got {tuple(scale.shape)} "
                            f"{scale.dtype}")
    return N, K


def save(path: str | os.PathLike, entries: dict[str, tuple[torch.Tensor, torch.Tensor]]) -> Path:
    """Writes {name: (tiles, scale)} to `path` (through a temporary file renamed into place)."""
    path = Path(path)
    header = {"format": FORMAT, "version": VERSION, "block": BLOCK, "layout": LAYOUT, "entries": {}}
    # Blob offsets depend on the header length, which depends on the offsets: size the header with
    # placeholder offsets of the final width first.
    raw = {name: (_bytes_of(t), _bytes_of(s)) for name, (t, s) in entries.items()}
    shapes = {name: _check_entry(name, t, s) for name, (t, s) in entries.items()}
    digests = {name: (hashlib.sha256(tb).hexdigest(), hashlib.sha256(sb).hexdigest()) for name, (tb, sb) in raw.items()}

    def build(offsets: dict[str, tuple[int, int]]) -> bytes:
        header["entries"] = {
            name: {"N": shapes[name][0], "K": shapes[name][1],
                   "tiles": {"offset": offsets[name][0], "nbytes": len(raw[name][0]), "sha256": digests[name][0]},
                   "scale": {"offset": offsets[name][1], "nbytes": len(raw[name][1]), "sha256": digests[name][1]}}
            for name in raw}
        return json.dumps(header, sort_keys=True).encode()

    big = 1 << 62
    probe = build({name: (big, big) for name in raw})
    cursor = _align(16 + len(probe) + 64)
    offsets = {}
    for name, (tb, sb) in raw.items():
        offsets[name] = (cursor, _align(cursor + len(tb)))
        cursor = _align(offsets[name][1] + len(sb))
    hdr = build(offsets)  # no longer than the probe: the real offsets have fewer digits

    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        for name, (tb, sb) in raw.items():
            for off, data in zip(offsets[name], (tb, sb)):
                f.seek(off)
                f.write(data)
        f.truncate(cursor)
    os.replace(tmp, path)
    return path


def read_header(path: str | os.PathLike) -> dict:
    """The JSON header of a tile-pack file, after the magic, version and blob-bounds checks."""
    path = Path(path)
    size = path.stat().st_size
    with open(path, "rb") as f:
        head = f.read(16)
        if len(head) != 16 or head[:8] != MAGIC:
            raise TilePackError(f"{path}: not a tile-pack file")
        (hlen,) = struct.unpack("<Q", head[8:])
        if hlen > size - 16:
            raise TilePackError(f"{path}: header length {hlen} past the end of the file")
        try:
            header = json.loads(f.read(hlen).decode())
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise TilePackError(f"{path}: unreadable header ({e})") from None
    if header.get("format") != FORMAT or header.get("version") != VERSION or header.get("block") != BLOCK:
        raise TilePackError(f"{path}: format {header.get('format')!r} v{header.get('version')} "
                            f"block {header.get('block')} is not {FORMAT} v{VERSION} block {BLOCK}")
    for name, e in header.get("entries", {}).items():
        N, K = e.get("N"), e.get("K")
        if not (isinstance(N, int) and isinstance(K, int) and N > 0 and K > 0 and N % BLOCK == 0 and K % BLOCK == 0):
            raise TilePackError(f"{path}: {name}: bad shape N={N} K={K}")
        want = {"tiles": N * K, "scale": 4 * (N // BLOCK) * (K // BLOCK)}
        for part, nbytes in want.items():
            blob = e.get(part, {})
            off, nb = blob.get("offset"), blob.get("nbytes")
            if nb != nbytes or not isinstance(off, int) or off % ALIGN or off < 16 + hlen or off + nb > size:
                raise TilePackError(f"{path}: {name}.{part}: offset {off} / {nb} bytes out of bounds or misaligned")
    return header


STAGE_BYTES = 32 << 20  # pinned staging chunk for loads to a GPU (two of them, alternating)


def load(path: str | os.PathLike, device: torch.device | str | None = None, names=None,
         verify: bool = False) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """Reads {name: (tiles uint8 [N/128, K/128, 128, 128], scale fp32 [N/128, K/128])} from `path`.

    device: where the tensors go. For a CUDA device the file is streamed through two pinned staging
    buffers, so reading one chunk overlaps the host-to-device copy of the previous one. names: a subset
    to read (KeyError for a name the file lacks). verify: check the stored SHA-256 of every blob read."""
    header = read_header(path)
    entries = header["entries"]
    wanted = list(entries) if names is None else list(names)
    dev = torch.device(device) if device is not None else torch.device("cpu")
    gpu = dev.type == "cuda"
    if gpu:
        stage = [torch.empty(STAGE_BYTES, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        done = [None, None]
        stream = torch.cuda.current_stream(dev)
        k = 0
    out = {}
    with open(path, "rb", buffering=0) as f:
        for name in wanted:
            e = entries[name]
            N, K = e["N"], e["K"]
            parts = []
            for part, shape, dtype in (("tiles", (N // BLOCK, K // BLOCK, BLOCK, BLOCK), torch.uint8),
                                       ("scale", (N // BLOCK, K // BLOCK), torch.float32)):
                blob = e[part]
                nbytes = blob["nbytes"]
                dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
                digest = hashlib.sha256() if verify else None
                f.seek(blob["offset"])
                for off in range(0, nbytes, STAGE_BYTES if gpu else nbytes):
                    n = min(STAGE_BYTES if gpu else nbytes, nbytes - off)
                    if gpu:
                        if done[k] is not None:
                            done[k].synchronize()  # the copy out of this staging buffer has finished
                        buf = stage[k][:n]
                    else:
                        buf = dst[off:off + n]
                    view = memoryview(buf.numpy())
                    got = 0
                    while got < n:
                        r = f.readinto(view[got:])
                        if not r:
                            raise TilePackError(f"{path}: {name}.{part}: short read ({off + got} of {nbytes} bytes)")
                        got += r
                    if digest is not None:
                        digest.update(view)
                    if gpu:
                        dst[off:off + n].copy_(buf, non_blocking=True)
                        done[k] = torch.cuda.Event()
                        done[k].record(stream)
                        k ^= 1
                if digest is not None and digest.hexdigest() != blob["sha256"]:
                    raise TilePackError(f"{path}: {name}.{part}: SHA-256 mismatch")
                parts.append(dst.view(dtype).view(shape))
            out[name] = (parts[0], parts[1])
    if gpu:
        stream.synchronize()
    return out

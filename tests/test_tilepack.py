"""CPU: the on-disk tile-first weight format (fp8_hand_b200/tilepack.py). The packed bytes come from the
oracle's restatement of the reference's tile-first permute (patches/fp8_hand_sm89.py:667)."""
import json
import struct

import pytest
import torch

from fp8_hand_b200 import tilepack
from oracle import oracle as O


def _entry(N, K, seed):
    w, s = O.make_weight(N, K, seed=seed)
    return O.relayout_tiles(w.view(torch.uint8)), s


def _sample(tmp_path):
    entries = {"mlp.gate_up_proj": _entry(512, 256, 1), "mlp.down_proj": _entry(256, 256, 2),
               "attn.o_proj": _entry(128, 384, 3)}
    return tilepack.save(tmp_path / "w.bsfp8", entries), entries


def test_round_trip_is_bit_exact(tmp_path):
    path, entries = _sample(tmp_path)
    got = tilepack.load(path, verify=True)
    assert set(got) == set(entries)
    for name, (tiles, scale) in entries.items():
        t, s = got[name]
        assert t.dtype == torch.uint8 and tuple(t.shape) == tuple(tiles.shape)
        assert torch.equal(t, tiles.view(torch.uint8)) and torch.equal(s, scale)


def test_tiles_are_the_reference_permute(tmp_path):
    """tiles[nb][kb][r][c] = W[nb*128 + r][kb*128 + c] for the stored bytes."""
    w, s = O.make_weight(256, 384, seed=9)
    path = tilepack.save(tmp_path / "w.bsfp8", {"w": (O.relayout_tiles(w.view(torch.uint8)), s)})
    t, _ = tilepack.load(path)["w"]
    W = w.view(torch.uint8)
    for nb, kb, r, c in [(0, 0, 0, 0), (1, 2, 127, 5), (0, 1, 64, 127), (1, 0, 3, 77)]:
        assert t[nb, kb, r, c] == W[nb * 128 + r, kb * 128 + c]


def test_layout_and_subset(tmp_path):
    path, entries = _sample(tmp_path)
    header = tilepack.read_header(path)
    assert header["format"] == "bsfp8-tiles" and header["version"] == 1 and header["block"] == 128
    for e in header["entries"].values():
        for part in ("tiles", "scale"):
            assert e[part]["offset"] % 4096 == 0
    got = tilepack.load(path, names=["mlp.down_proj"])
    assert list(got) == ["mlp.down_proj"]
    with pytest.raises(KeyError):
        tilepack.load(path, names=["missing"])


def test_rejects_bad_files(tmp_path):
    path, _ = _sample(tmp_path)
    raw = bytearray(path.read_bytes())

    bad = tmp_path / "magic.bsfp8"
    bad.write_bytes(b"NOTATILE" + bytes(raw[8:]))
    with pytest.raises(tilepack.TilePackError):
        tilepack.read_header(bad)

    short = tmp_path / "short.bsfp8"
    short.write_bytes(bytes(raw[: len(raw) // 2]))
    with pytest.raises(tilepack.TilePackError):
        tilepack.read_header(short)

    # a blob offset that is not 4096-aligned
    (hlen,) = struct.unpack("<Q", bytes(raw[8:16]))
    header = json.loads(bytes(raw[16:16 + hlen]))
    name = next(iter(header["entries"]))
    header["entries"][name]["scale"]["offset"] += 8
    hdr = json.dumps(header, sort_keys=True).encode()
    assert len(hdr) <= hlen
    moved = tmp_path / "moved.bsfp8"
    moved.write_bytes(bytes(raw[:8]) + struct.pack("<Q", len(hdr)) + hdr + bytes(raw[16 + len(hdr):]))
    with pytest.raises(tilepack.TilePackError):
        tilepack.read_header(moved)

    # a flipped tile byte: accepted without verify, caught with it
    e = tilepack.read_header(path)["entries"][name]
    raw[e["tiles"]["offset"] + 17] ^= 0xFF
    flipped = tmp_path / "flipped.bsfp8"
    flipped.write_bytes(bytes(raw))
    tilepack.load(flipped, names=[name])
    with pytest.raises(tilepack.TilePackError):
        tilepack.load(flipped, names=[name], verify=True)


def test_save_checks_shapes(tmp_path):
    tiles, scale = _entry(256, 256, 4)
    with pytest.raises(tilepack.TilePackError):
        tilepack.save(tmp_path / "x.bsfp8", {"w": (tiles.view(-1), scale)})
    with pytest.raises(tilepack.TilePackError):
        tilepack.save(tmp_path / "x.bsfp8", {"w": (tiles, scale[:1])})
    with pytest.raises(tilepack.TilePackError):
        tilepack.save(tmp_path / "x.bsfp8", {"w": (tiles, scale.double())})

"""Snapshot file plumbing that needs no GPU: the header check and the two readers."""

from __future__ import annotations

import json
import os

import pytest
import torch

from lazykv_b200 import snapshot


def _write(path, sections: list[torch.Tensor], magic: str = snapshot.MAGIC) -> dict:  # noqa: ANN001
    """A file in the snapshot layout: header, then each section at an ALIGN-padded offset."""
    offsets, cursor = {}, 0
    for i, t in enumerate(sections):
        offsets[f"s{i}"] = [cursor, t.numel() * t.element_size()]
        cursor += snapshot._pad(offsets[f"s{i}"][1])
    head = json.dumps({"magic": magic, "sections": offsets}).encode()
    base = snapshot._pad(len(head) + 8)
    with path.open("wb") as f:
        f.write(len(head).to_bytes(8, "little") + head)
        f.write(b"\0" * (base - len(head) - 8))
        for t in sections:
            n = f.write(snapshot._bytes(t))
            f.write(b"\0" * (snapshot._pad(n) - n))
    return offsets


def test_header_accepts_both_magics_and_refuses_foreign_files(tmp_path) -> None:  # noqa: ANN001
    for magic in (snapshot.MAGIC, snapshot.MAGIC_INT8):
        p = tmp_path / f"{magic}.lkv"
        _write(p, [torch.zeros(3)], magic)
        header, base = snapshot.read_header(p)
        assert header["magic"] == magic and base % snapshot.ALIGN == 0
    bad = tmp_path / "bad.lkv"
    bad.write_bytes((2).to_bytes(8, "little") + b"{}")
    with pytest.raises(ValueError, match="not a LazyKV snapshot"):
        snapshot.read_header(bad)


def test_sections_are_aligned_and_both_readers_return_their_bytes(tmp_path) -> None:  # noqa: ANN001
    gen = torch.Generator().manual_seed(0)
    # sizes around the alignment and a reader chunk edge, a bf16 section (no numpy dtype)
    secs = [torch.randint(0, 255, (n,), generator=gen, dtype=torch.uint8) for n in (1, 4095, 4096, 4097)]
    secs.append(torch.randn((3, 5, 7), generator=gen).bfloat16())
    p = tmp_path / "s.lkv"
    offsets = _write(p, secs)
    header, base = snapshot.read_header(p)
    assert all(o % snapshot.ALIGN == 0 for o, _ in offsets.values())
    assert os.path.getsize(p) % snapshot.ALIGN == 0
    with p.open("rb", buffering=0) as f:
        for i, t in enumerate(secs):
            out = torch.empty_like(t)
            snapshot._read_into(f, base + offsets[f"s{i}"][0], out)
            assert torch.equal(out, t)
    try:
        reader = snapshot._DirectReader(p)
    except OSError as e:  # a filesystem without O_DIRECT (tmpfs, some overlays)
        pytest.skip(f"no O_DIRECT here: {e}")
    try:
        reader.CHUNK = 8192  # several chunks per section
        for i, t in enumerate(secs):
            out = torch.empty_like(t)
            reader.read_into(base + offsets[f"s{i}"][0], out)
            assert torch.equal(out, t)
    finally:
        reader.close()

"""Session snapshots: a tiered session's KV saved to disk and resumed without a prefill.

API and file layout of lazykv/snapshot.py (save :72-123, read_header :126-133, restore :187-278),
extended to the int8 tier, which the reference refuses.

A sealed block never changes once it is in the pinned host store, so a snapshot is that store as
it is, plus what is only on the GPU: the dense layers' KV, each tiered layer's unsealed tail and
the logits for the next token. Restore reads each tiered layer's blocks straight into its pinned
store and derives the metadata and the seeded slots from those bytes on the device
(`TieredLayer.from_store`), so a restored tier is the tier the constructor builds at that length;
only slot residency, which decides what is fetched and never what is attended, starts afresh.

File: a JSON header (its length as 8 little-endian bytes first) padded to `ALIGN`, then sections,
each at a multiple of `ALIGN`: the next-token logits (float32), then per layer either `[2, h, L, d]`
(dense layers: keys, values) or the store's own blocks followed by the `[h, 2, fill, d]` tail
(tiered layers). A bf16 tier's blocks are `[n, h, 2, bs, d]` and its file is the reference's format
(same magic, header keys and section names), so either side reads the other's. An int8 tier's file
has its own magic (a reader of the bf16 format rejects it rather than misreading it), `"quant":
"int8"` and `"record_bytes"` in the header, the records `[n, h, W]` as `L{i}.records`, and
`L{i}.sink`, the exact first block `[h, 2, bs, d]` that stays in VRAM (its record is lossy).
"""

from __future__ import annotations

import json
import mmap
import os
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, BinaryIO

import torch

from lazykv_b200.cache import FullGPUCache
from lazykv_b200.pinned import pinned_empty
from lazykv_b200.quant import packed_pair_bytes
from lazykv_b200.tiered import TieredCache, TieredLayer

MAGIC = "lazykv-snapshot-1"
MAGIC_INT8 = "lazykv-snapshot-1+int8"
ALIGN = 4096  # page and sector size: what an unbuffered (O_DIRECT) reader needs
_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _pad(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


def _bytes(t: torch.Tensor) -> memoryview:
    """A CPU tensor's bytes, without a copy for a contiguous one (bfloat16 has no numpy dtype)."""
    t = t.contiguous()
    return memoryview(t.view(torch.uint8).reshape(-1).numpy())


@dataclass
class SaveStats:
    bytes_written: int
    seconds: float  # including fsync: the snapshot is on disk when save returns


@dataclass
class RestoreStats:
    bytes_read: int
    read_s: float
    rebuild_s: float  # everything outside reads: allocation, H2D, metadata, seeding, dense layers, the final sync
    sections: dict[str, float] = field(default_factory=dict)


def save(cache: TieredCache, next_logits: torch.Tensor, path: Path) -> SaveStats:
    """Write `cache` (a tiered session at any decode position) and the logits for its next token."""
    t0 = time.perf_counter()
    torch.cuda.synchronize()  # seals copy and pack into the store asynchronously
    tiers = cache.tiers
    any_tier = next(iter(tiers.values()))
    length = any_tier.length
    int8 = cache.quant is not None
    sections: list[tuple[str, torch.Tensor]] = [("logits", next_logits.float().cpu())]
    layers: list[dict[str, Any]] = []
    for i in range(len(cache.full.layers)):
        if i in tiers:
            t = tiers[i]
            if t.length != length:
                raise RuntimeError("tiered layers disagree on length")
            tail = t.pool[t.tail_slot, :, :, : t.fill].cpu()  # [h, 2, fill, d]
            if int8:
                sections.append((f"L{i}.records", t.host[: t.n_sealed]))
                sections.append((f"L{i}.sink", t.pool[0].cpu()))
            else:
                sections.append((f"L{i}.blocks", t.host[: t.n_sealed]))
            sections.append((f"L{i}.tail", tail))
            layers.append({"kind": "tier", "n_sealed": t.n_sealed, "fill": t.fill})
        else:
            src = cache.full.layers[i]
            if src.get_seq_length() != length:
                raise RuntimeError(f"dense layer {i} has length {src.get_seq_length()}, the tier {length}")
            kv = torch.stack([src.keys[0, :, :length], src.values[0, :, :length]]).cpu()  # [2, h, L, d]
            sections.append((f"L{i}.kv", kv))
            layers.append({"kind": "dense"})
    offsets, cursor = {}, 0
    for name, t in sections:
        offsets[name] = [cursor, t.numel() * t.element_size()]
        cursor += _pad(offsets[name][1])
    header: dict[str, Any] = {
        "magic": MAGIC_INT8 if int8 else MAGIC, "length": length, "block_size": cache.block_size, "dense_layers": cache.dense_layers,
        "heads": any_tier.h, "head_dim": any_tier.d, "dtype": str(any_tier.pool.dtype).removeprefix("torch."),
        "vocab": int(next_logits.numel()), "layers": layers, "sections": offsets,
    }
    if int8:
        header["quant"] = "int8"
        header["record_bytes"] = packed_pair_bytes(any_tier.bs, any_tier.d)
    head = json.dumps(header).encode()
    base = _pad(len(head) + 8)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("wb") as f:
        f.write(len(head).to_bytes(8, "little") + head)
        f.write(b"\0" * (base - len(head) - 8))
        for _, t in sections:
            n = f.write(_bytes(t))
            f.write(b"\0" * (_pad(n) - n))
        f.flush()
        os.fsync(f.fileno())
    return SaveStats(base + cursor, time.perf_counter() - t0)


def read_header(path: Path) -> tuple[dict[str, Any], int]:
    """The header and the file offset where the sections start."""
    with path.open("rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
    if header.get("magic") not in (MAGIC, MAGIC_INT8):
        raise ValueError(f"{path} is not a LazyKV snapshot")
    return header, _pad(n + 8)


def _read_into(f: BinaryIO, offset: int, out: torch.Tensor) -> None:
    f.seek(offset)
    view = _bytes(out)  # `out` is contiguous, so this aliases its memory
    got = f.readinto(view)
    if got != len(view):
        raise EOFError(f"short read: {got} of {len(view)} bytes at offset {offset}")


class _DirectReader:
    """Reads that bypass the page cache (O_DIRECT), the Linux counterpart of the reference's
    Windows FILE_FLAG_NO_BUFFERING reader (snapshot.py:136-184).

    Without it, a snapshot read back soon after it was written comes from RAM and its "disk" time
    is a memcpy. O_DIRECT needs aligned offsets, sizes and buffers: `save` aligns and pads every
    section, and the reads land in a page-aligned anonymous mapping and are copied out from there.
    """

    CHUNK = 64 * 2**20

    def __init__(self, path: Path) -> None:
        try:
            self._fd = os.open(path, os.O_RDONLY | os.O_DIRECT)
        except OSError as e:
            raise OSError(e.errno, f"cannot open {path} for unbuffered reads (O_DIRECT): {e.strerror}") from e
        self._buf = mmap.mmap(-1, self.CHUNK)
        self._view = torch.frombuffer(self._buf, dtype=torch.uint8)

    def read_into(self, offset: int, out: torch.Tensor) -> None:
        dst = out.view(torch.uint8).reshape(-1)
        n, done = dst.numel(), 0
        while done < n:
            want = min(self.CHUNK, _pad(n - done))
            try:
                got = os.preadv(self._fd, [memoryview(self._buf)[:want]], offset + done)
            except OSError as e:
                raise OSError(e.errno, f"unbuffered read failed at offset {offset + done}: {e.strerror}") from e
            take = min(got, n - done)
            if take <= 0:
                raise EOFError(f"short unbuffered read at offset {offset + done}")
            dst[done : done + take].copy_(self._view[:take])
            done += take

    def close(self) -> None:
        del self._view
        self._buf.close()
        os.close(self._fd)


def restore(path: Path, k_blocks: int, capacity_tokens: int, num_layers: int, model: Any = None, host_pools: list[torch.Tensor] | None = None,
            n_slots: int | None = None, fetch: str = "gather", stages: Any = None, unbuffered: bool = False, rebuild: str = "store",
            cold_placement: str = "host", cache_cls: type[TieredCache] = TieredCache) -> tuple[TieredCache, torch.Tensor, RestoreStats]:
    """A cache at the snapshot's position (a `cache_cls`, TieredCache by default) and the logits for
    its next token.

    By default reads go through the OS page cache; `unbuffered=True` reads from the disk itself
    (O_DIRECT, Linux), which is what a resumed session pays once the cache has moved on. `rebuild`:
    "store" reads the sealed blocks straight into each layer's pinned store and derives the rest on
    the device without a host sync, so that work overlaps the next layer's read; "boundary" (bf16
    only) copies each layer to the GPU and hands it to the constructor, the tiered-prefill boundary.
    Both give the same state.
    """
    if rebuild not in ("store", "boundary"):
        raise ValueError(f"unknown rebuild {rebuild!r}")
    if unbuffered and not hasattr(os, "O_DIRECT"):
        raise NotImplementedError("unbuffered reads need O_DIRECT (Linux)")
    header, base = read_header(path)
    quant = header.get("quant")
    if quant is not None and rebuild == "boundary":
        raise ValueError("an int8 snapshot holds records, not the exact KV the constructor takes: use rebuild='store'")
    dt = _DTYPES[header["dtype"]]
    h, d, bs, length = header["heads"], header["head_dim"], header["block_size"], header["length"]
    if len(header["layers"]) != num_layers:
        raise ValueError(f"snapshot has {len(header['layers'])} layers, the model {num_layers}")
    sec = header["sections"]
    stats = RestoreStats(0, 0.0, 0.0)
    dev = torch.device("cuda")
    full = FullGPUCache(num_layers, capacity_tokens)
    tiers: dict[int, TieredLayer] = {}
    dense = 0
    reader = _DirectReader(path) if unbuffered else None
    try:
        with path.open("rb", buffering=0) as f:

            def load(name: str, shape: tuple[int, ...], dtype: torch.dtype, into: torch.Tensor | None = None) -> torch.Tensor:
                out = torch.empty(shape, dtype=dtype) if into is None else into
                if out.numel() * out.element_size() != sec[name][1]:
                    raise ValueError(f"section {name} holds {sec[name][1]} bytes, expected {out.numel() * out.element_size()}")
                t0 = time.perf_counter()
                if reader is not None:
                    reader.read_into(base + sec[name][0], out)
                else:
                    _read_into(f, base + sec[name][0], out)
                dt_s = time.perf_counter() - t0
                stats.read_s += dt_s
                stats.sections[name] = dt_s
                stats.bytes_read += sec[name][1]
                return out

            logits = load("logits", (header["vocab"],), torch.float32).to(dev)
            for i, spec in enumerate(header["layers"]):
                if spec["kind"] == "dense":
                    kv = load(f"L{i}.kv", (2, h, length, d), dt)
                    t0 = time.perf_counter()
                    g = kv.to(dev)
                    full.layers[i].update(g[0:1], g[1:2])
                    stats.rebuild_s += time.perf_counter() - t0
                    dense += 1
                    continue
                n, fill = spec["n_sealed"], spec["fill"]
                host = None if host_pools is None else host_pools[i - header["dense_layers"]]
                if rebuild == "store":
                    t0 = time.perf_counter()
                    cap = -(-capacity_tokens // bs)
                    if host is None:
                        shape = (cap, h, 2, bs, d) if quant is None else (cap, h, header["record_bytes"])
                        host = pinned_empty(shape, dt if quant is None else torch.uint8)
                    stats.rebuild_s += time.perf_counter() - t0
                    if quant is None:
                        load(f"L{i}.blocks", (n, h, 2, bs, d), dt, into=host[:n])
                        sink = None
                    else:
                        load(f"L{i}.records", (n, h, header["record_bytes"]), torch.uint8, into=host[:n])
                        sink = load(f"L{i}.sink", (h, 2, bs, d), dt)
                    tail = load(f"L{i}.tail", (h, 2, fill, d), dt)
                    t0 = time.perf_counter()
                    tiers[i] = TieredLayer.from_store(host, n, tail, k_blocks, bs, capacity_tokens, dev, n_slots, quant=quant, sink=sink,
                                                      cold_placement=cold_placement)
                    stats.rebuild_s += time.perf_counter() - t0
                    continue
                blocks = load(f"L{i}.blocks", (n, h, 2, bs, d), dt)
                tail = load(f"L{i}.tail", (h, 2, fill, d), dt)
                t0 = time.perf_counter()
                g = blocks.to(dev).permute(1, 2, 0, 3, 4).reshape(h, 2, n * bs, d)  # [h, 2, n*bs, d]
                kv = torch.cat([g, tail.to(dev)], dim=2)
                tiers[i] = TieredLayer(kv[None, :, 0], kv[None, :, 1], k_blocks, bs, capacity_tokens, host, n_slots, cold_placement=cold_placement)
                del g, kv
                stats.rebuild_s += time.perf_counter() - t0
    finally:
        if reader is not None:
            reader.close()
    if dense != header["dense_layers"]:
        raise ValueError("snapshot's dense layer count disagrees with its header")
    t0 = time.perf_counter()
    cache = cache_cls(full, k_blocks, bs, capacity_tokens, model=model, dense_layers=dense, n_slots=n_slots, fetch=fetch, stages=stages,
                      tiers=tiers, quant=quant, cold_placement=cold_placement)
    torch.cuda.synchronize()
    stats.rebuild_s += time.perf_counter() - t0
    return cache, logits, stats

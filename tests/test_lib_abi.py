"""The C-ABI library loads without a GPU, exports every entry point include/lkv.h declares, and
rejects invalid arguments with a status and a message before touching the device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "lkv.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(lkv_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from lazykv_b200 import _lib

    if not _lib.LIB_PATH.exists():
        from lazykv_b200.build import build

        build()
    return _lib.lib()


def test_every_declared_entry_point_is_exported_and_bound(lib) -> None:  # noqa: ANN001
    from lazykv_b200 import _lib

    names = declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version_and_record_width(lib) -> None:  # noqa: ANN001
    assert lib.lkv_version().startswith(b"lkv_sm100")
    assert lib.lkv_packed_pair_bytes(16, 64) == 2368
    assert lib.lkv_packed_pair_bytes(64, 64) == 8704


def test_invalid_arguments_return_a_status_and_a_message(lib) -> None:  # noqa: ANN001
    from lazykv_b200 import _lib

    # k larger than the candidates: rejected before any launch.
    rc = lib.lkv_quest_topk(None, 1, 32, 8, 64, None, None, 1, 0, 1, 10, 11, 1, 0, None, 11, None, None, 0, None, 0, None)
    assert rc == 1 and "k <= n_cand" in _lib.last_error()
    rc = lib.lkv_quest_topk(None, 1, 30, 8, 64, None, None, 1, 0, 1, 10, 5, 1, 0, None, 5, None, None, 0, None, 0, None)
    assert rc == 1 and "do not group" in _lib.last_error()
    rc = lib.lkv_pack_int8(None, 1, 1, 8, 12, 64, None, None, None, 0, 0, None, None)
    assert rc == 1 and "geometry" in _lib.last_error()
    rc = lib.lkv_hot_attention(None, 32, 8, 64, 16, None, None, 1, 0, 0, 0, 0, None, 4, None, 0, 0, 0.125, None, None, None, 0, None)
    assert rc == 2 and "null" in _lib.last_error()
    rc = lib.lkv_lse_merge(None, None, 0, 4, 64, None, 0, None, None)
    assert rc == 1
    # first-pass counters (64 heads x 256), the selection's failure words (64 heads), then the keys
    assert lib.lkv_quest_topk_workspace(8, 8190) == 64 * 1024 + 256 + 8 * 8190 * 8
    assert lib.lkv_attention_workspace(8, 32, 64, 2048) > 0
    buf = ctypes.create_string_buffer(4)
    assert lib.lkv_last_error(buf, 4) > 3 and len(buf.value) == 3


def test_the_append_mark_and_stage_entries_reject_bad_arguments(lib) -> None:  # noqa: ANN001
    """lkv_append_tokens, lkv_mark_blocks and lkv_ragged_stage_records validate before any launch."""
    from lazykv_b200 import _lib

    fake = ctypes.c_void_p(16)  # never dereferenced: every call below fails its checks first
    # 3 tokens at fill 14 overrun a block of 16
    rc = lib.lkv_append_tokens(fake, 64, 64, fake, 64, 64, 8, 3, 64, _lib.LKV_BF16, fake, 16, 14, None)
    assert rc == 1 and "do not fit" in _lib.last_error()
    rc = lib.lkv_append_tokens(None, 64, 64, fake, 64, 64, 8, 1, 64, _lib.LKV_BF16, fake, 16, 0, None)
    assert rc == 2 and "null" in _lib.last_error()
    rc = lib.lkv_append_tokens(fake, 64, 64, fake, 64, 64, 8, 1, 64, 7, fake, 16, 0, None)
    assert rc == 1 and "dtype" in _lib.last_error()
    # a row stride below k; a null bitmap
    rc = lib.lkv_mark_blocks(fake, 8, 10, 5, fake, 4, None)
    assert rc == 1 and "ids_ld >= k" in _lib.last_error()
    rc = lib.lkv_mark_blocks(fake, 8, 10, 10, None, 4, None)
    assert rc == 2 and "null" in _lib.last_error()
    # a record width that is not a multiple of 16; a misaligned stage
    rc = lib.lkv_ragged_stage_records(fake, 10, 8, 2360, fake, 9, fake, 1, fake, None, 0, fake, 10, fake, fake, 9, None)
    assert rc == 1 and "bad shape" in _lib.last_error()
    rc = lib.lkv_ragged_stage_records(fake, 10, 8, 2368, fake, 9, fake, 1, fake, None, 0, ctypes.c_void_p(24), 10, fake, fake, 9, None)
    assert rc == 2 and "16-byte aligned" in _lib.last_error()


def test_the_split_step_entries_reject_missing_arguments(lib) -> None:  # noqa: ANN001
    """lkv_split_step and its events API refuse null handles before touching a stream."""
    from lazykv_b200 import _lib

    assert lib.lkv_split_events_create(None) == 2 and "null" in _lib.last_error()
    assert lib.lkv_split_step(None, None, None, None) == 2 and "null" in _lib.last_error()
    assert lib.lkv_split_join(None, None) == 2 and "null" in _lib.last_error()
    assert lib.lkv_split_wait(None) == 2 and "null" in _lib.last_error()
    assert lib.lkv_split_events_destroy(None) == 0
    assert ctypes.sizeof(_lib.SplitStepArgs) == 336  # the C struct's size on this ABI (x86-64)

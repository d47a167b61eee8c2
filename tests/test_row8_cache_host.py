"""Host logic of the row8 pack cache (cached_pack_weight_rows8): budget
parsing, hits, least-recently-used eviction and the statistics keys that
the reference's callers read (src/pcketlm/native/__init__.py:2110-2193).
The GPU pack itself is replaced by a CPU stand-in of the same size."""

import torch

from pocketlm_b200 import native


def _fake_pack(weight):
    return torch.zeros((weight.numel(),), dtype=torch.uint16)


def test_budget_parsing(monkeypatch):
    for text, want in (("", 0), ("abc", 0), ("-4", 0), ("0", 0), (" 3 ", 3 << 20), ("+2", 2 << 20)):
        monkeypatch.setenv("PCKETLM_PACKED_GEMV_CACHE_MB", text)
        assert native.packed_gemv_cache_stats()["budget_bytes"] == want


def test_hits_evictions_and_oversize(monkeypatch):
    monkeypatch.setattr(native, "pack_weight_rows8", _fake_pack)
    monkeypatch.setenv("PCKETLM_PACKED_GEMV_CACHE_MB", "1")
    native.reset_packed_gemv_cache()
    quarter = torch.zeros((1 << 18,), dtype=torch.float16).view(512, 512)  # 512 KiB pack: two fit in 1 MiB
    a = native.cached_pack_weight_rows8("a", quarter)
    b = native.cached_pack_weight_rows8("b", quarter)
    assert native.cached_pack_weight_rows8("a", quarter) is a  # a is now the most recent
    c = native.cached_pack_weight_rows8("c", quarter)  # evicts b, the least recently used
    st = native.packed_gemv_cache_stats()
    assert (st["hits"], st["misses"], st["stores"], st["evictions"]) == (1, 3, 3, 1)
    assert st["resident_count"] == 2 and st["resident_bytes"] == 2 * (512 << 10) and st["resident_mb"] == 1.0
    assert native.cached_pack_weight_rows8("c", quarter) is c
    assert native.cached_pack_weight_rows8("b", quarter) is not b  # b was evicted: packed again
    big = torch.zeros((1 << 20,), dtype=torch.float16).view(1024, 1024)  # 2 MiB > budget: returned, not kept
    native.cached_pack_weight_rows8("big", big)
    st = native.packed_gemv_cache_stats()
    assert st["resident_count"] == 2 and st["stores"] == 4
    native.reset_packed_gemv_cache()
    assert native.packed_gemv_cache_stats()["resident_count"] == 0


def test_disabled_and_zero_budget_do_not_keep(monkeypatch):
    monkeypatch.setattr(native, "pack_weight_rows8", _fake_pack)
    w = torch.zeros((8, 8), dtype=torch.float16)
    for env in ({"PCKETLM_PACKED_GEMV_CACHE_MB": "0"},
                {"PCKETLM_PACKED_GEMV_CACHE_MB": "8", "PCKETLM_DISABLE_PACKED_GEMV_CACHE": "1"}):
        native.reset_packed_gemv_cache()
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        first = native.cached_pack_weight_rows8("w", w)
        assert native.cached_pack_weight_rows8("w", w) is not first
        st = native.packed_gemv_cache_stats()
        assert st["misses"] == 2 and st["hits"] == 0 and st["resident_count"] == 0
        monkeypatch.delenv("PCKETLM_DISABLE_PACKED_GEMV_CACHE", raising=False)
    native.reset_packed_gemv_cache()

"""The tuner's bookkeeping on the host (no GPU): a run that tunes some shapes
must save every entry of the tuned-config file, not only the shapes it timed.

The timing itself (tune_gemv) and the device queries are stubbed; what is
tested is the load / update / save path of `python -m roofline_decoding_b200.tuner`.
"""
import json

import pytest

from roofline_decoding_b200 import kernels, tuner
from roofline_decoding_b200._lib import GemvConfig


@pytest.fixture
def isolated_cache(monkeypatch, tmp_path):
    """A tuned-config file of two entries, and a fresh in-memory cache."""
    src = tmp_path / "tuned.json"
    entries = [
        {"key": ["NVIDIA B200", 1, 8192, 28672, "float16", 0, 0], "config": [4, 1, 4, 3, 0]},
        {"key": ["NVIDIA B200", 1, 1536, 1536, "float16", 0, 0], "config": [4, 2, 2, 6, 0]},
    ]
    src.write_text(json.dumps({"entries": entries}))
    monkeypatch.setenv("W4B200_TUNED_CONFIGS", str(src))
    monkeypatch.setattr(kernels, "_TUNE_CACHE", {})
    monkeypatch.setattr(kernels, "_loaded_tuned_file", False)
    monkeypatch.setattr(kernels, "_device_key", lambda device: "NVIDIA B200")
    monkeypatch.setattr(kernels, "default_config", lambda *a, **k: GemvConfig(1, 8, 2, 1, 0))
    monkeypatch.setattr(tuner.torch.cuda, "current_device", lambda: 0)

    def fake_tune(M, K, N, x_dtype, y_dtype, split_k, num_warps, device, return_table=False,
                  streaming=True):
        # large N: a streaming grid wins unless one tile per CTA is asked for
        best = GemvConfig(1, 8, 4, 2, 0, 148) if N >= 28672 and streaming else GemvConfig(1, 8, 2, 1, 0)
        table = [(2.5, best.as_tuple())]
        return (best, table) if return_table else best

    monkeypatch.setattr(tuner, "tune_gemv", fake_tune)
    return tmp_path


def test_quick_run_keeps_the_shapes_it_does_not_tune(isolated_cache):
    out = isolated_cache / "out.json"
    tuner.main(["--quick", "--dtypes", "fp16", "--out", str(out)])
    saved = {tuple(e["key"]): e["config"] for e in json.loads(out.read_text())["entries"]}
    # the large shape was not in the quick set: it must survive the save
    assert saved[("NVIDIA B200", 1, 8192, 28672, "float16", 0, 0)] == [4, 1, 4, 3, 0]
    # a tuned shape takes the new winner
    assert saved[("NVIDIA B200", 1, 1536, 1536, "float16", 0, 0)] == [1, 8, 2, 1, 0]
    # and every quick shape is present
    for M, K, N in tuner.WORKLOAD_SHAPES[:8]:
        assert ("NVIDIA B200", M, K, N, "float16", 0, 0) in saved


def test_save_and_reload_round_trip(isolated_cache):
    kernels._load_tuned_file()
    path = kernels.save_tuned_configs(isolated_cache / "round.json")
    rows = json.loads(path.read_text())["entries"]
    assert len(rows) == 2
    assert all(len(r["config"]) == 5 for r in rows)


def test_one_tile_requests_never_get_a_streaming_grid(isolated_cache):
    """Epilogues and the peer gather need one column tile per CTA: a streaming
    winner is replaced by the stored one-tile winner, else by the default
    tile (no tuning allowed) or by a one-tile tuning run."""
    import torch

    kernels._load_tuned_file()
    key = ("NVIDIA B200", 1, 8192, 28672, "float16", 0, 0)
    kernels._TUNE_CACHE[key] = (1, 8, 4, 2, 0, 148)
    get = lambda **kw: kernels.tuned_config(1, 8192, 28672, torch.float16, torch.float16,  # noqa: E731
                                            None, None, "cpu", **kw)
    assert get().columns == 148
    assert get(streaming=False, tune=False).as_tuple() == (1, 8, 2, 1, 0)  # the default
    kernels._TUNE_CACHE[key + ("one_tile",)] = (2, 4, 5, 1, 0)
    assert get(streaming=False).as_tuple() == (2, 4, 5, 1, 0)
    # a one-tile winner serves both requests
    key2 = ("NVIDIA B200", 1, 1536, 1536, "float16", 0, 0)
    assert kernels.tuned_config(1, 1536, 1536, torch.float16, torch.float16, None, None, "cpu",
                                streaming=False).as_tuple() == (4, 2, 2, 6, 0)
    assert key2 + ("one_tile",) not in kernels._TUNE_CACHE


def test_tuner_stores_the_one_tile_winner_beside_a_streaming_one(isolated_cache, monkeypatch):
    out = isolated_cache / "out.json"
    tuner.main(["--dtypes", "fp16", "--out", str(out)])
    saved = {tuple(e["key"]): e["config"] for e in json.loads(out.read_text())["entries"]}
    key = ("NVIDIA B200", 1, 8192, 28672, "float16", 0, 0)
    assert saved[key] == [1, 8, 4, 2, 0, 148]
    assert saved[key + ("one_tile",)] == [1, 8, 2, 1, 0]
    assert ("NVIDIA B200", 1, 1536, 1536, "float16", 0, 0, "one_tile") not in saved
    # and the file loads back with both entries
    kernels._TUNE_CACHE.clear()
    kernels._loaded_tuned_file = False
    monkeypatch.setenv("W4B200_TUNED_CONFIGS", str(out))
    kernels._load_tuned_file()
    assert kernels._TUNE_CACHE[key + ("one_tile",)] == (1, 8, 2, 1, 0)

"""Session files in the reference's layout (kandiga/engine.py:1342-1479): an
npz of cache_{i}_{j} arrays (16-bit dtypes as uint16 bit patterns) plus a
_meta.json with history, tokens_fed, model, dtype_map and layer_info.  CPU
part: plain [keys, values] layers round-trip bit-exactly."""
import json

import numpy as np
import pytest
import torch

from kandiga_b200.kv_compress import load_session, save_session


def test_kv_layers_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    layers = [
        [torch.randn(1, 2, 5, 64, generator=g).half(), torch.randn(1, 2, 5, 64, generator=g).half()],
        None,  # a layer without a cache is skipped
        [torch.randn(1, 4, 3, 128, generator=g).bfloat16(), torch.randn(1, 4, 3, 128, generator=g).bfloat16()],
        [torch.randn(2, 1, 7, 64, generator=g), torch.randn(2, 1, 7, 64, generator=g)],
    ]
    path = str(tmp_path / "s.npz")
    save_session(path, layers, history=[{"role": "user", "content": "hi"}], tokens_fed=15, model="m")
    meta = json.load(open(str(tmp_path / "s_meta.json")))
    assert meta["tokens_fed"] == 15 and meta["model"] == "m" and meta["history"][0]["content"] == "hi"
    assert set(meta["layer_info"]) == {"0", "2", "3"}
    assert meta["layer_info"]["2"] == {"type": "KVCache", "n": 2, "offset": 3}
    assert meta["dtype_map"]["cache_2_0"] == {"shape": [1, 4, 3, 128], "dtype": "bfloat16"}
    raw = np.load(path)
    assert raw["cache_0_0"].dtype == np.uint16 and raw["cache_3_1"].dtype == np.float32
    got, meta2 = load_session(path, model="m", device="cpu")
    assert got[1] is None
    for i in (0, 2, 3):
        for a, b in zip(layers[i], got[i]):
            assert a.dtype == b.dtype and torch.equal(a, b)
    with pytest.raises(ValueError):
        load_session(path, model="other", device="cpu")

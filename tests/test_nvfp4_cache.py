"""Load-time NVFP4 packing with its on-disk cache (nvfp4_dense.py; the reference's
nvfp4_dense.py in patches/sglang/series/0095-…patch:90-200), on the CPU: packs from the
checkpoint's own rows (bit-identical to the oracle's quantiser, which is pinned to the
reference's), finds the shard through the index json or by scanning headers, reuses the
cached file on the second call, keys on the row set and the shard's identity, and leaves
no temporary file behind."""

import json
import os

import numpy as np
import pytest
import torch

from flash_next_rtxpro6000_b200 import nvfp4_dense as nd
from oracle import nvfp4 as onv


@pytest.fixture()
def model_dir(tmp_path):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(3)
    head = (torch.randn(96, 256, generator=g) * 0.05).bfloat16()
    other = torch.randn(8, 8, generator=g).bfloat16()
    d = tmp_path / "model"
    d.mkdir()
    save_file({"model.norm.weight": other}, str(d / "model-00001-of-00002.safetensors"))
    save_file({"lm_head.weight": head}, str(d / "model-00002-of-00002.safetensors"))
    return d, head


def _expected(w):
    wq, bs, gs = onv.quantize(w.float().numpy())
    return wq, bs, gs


@pytest.mark.parametrize("with_index", [False, True])
def test_pack_cache_and_reuse(model_dir, tmp_path, monkeypatch, with_index):
    d, head = model_dir
    if with_index:
        (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {
            "lm_head.weight": "model-00002-of-00002.safetensors",
            "model.norm.weight": "model-00001-of-00002.safetensors"}}))
    assert nd.find_shard(str(d), "lm_head.weight").endswith("model-00002-of-00002.safetensors")
    cache = tmp_path / "cache"
    wq, bs, gs = nd.build_or_load(str(d), "lm_head.weight", device="cpu", cache_dir=str(cache))
    ewq, ebs, egs = _expected(head)
    assert np.array_equal(wq.numpy(), ewq) and np.array_equal(bs.numpy(), ebs)
    assert np.array_equal(gs.numpy().reshape(-1), np.asarray(egs).reshape(-1))
    files = os.listdir(cache)
    assert len(files) == 1 and ".tmp" not in files[0]

    def no_read(*a, **k):
        raise AssertionError("the cached weight must be reused")

    monkeypatch.setattr(nd, "read_rows", no_read)
    wq2, bs2, gs2 = nd.build_or_load(str(d), "lm_head.weight", device="cpu", cache_dir=str(cache))
    assert torch.equal(wq2, wq) and torch.equal(bs2, bs) and torch.equal(gs2, gs)


def test_row_subset_and_key_changes(model_dir, tmp_path):
    d, head = model_dir
    rows = torch.tensor([5, 0, 77, 31, 90, 2, 64, 13], dtype=torch.int64)
    cache = tmp_path / "cache"
    k_all = nd.cache_key(str(d), "lm_head.weight", None)
    k_rows = nd.cache_key(str(d), "lm_head.weight", rows)
    assert k_all != k_rows
    assert nd.cache_key(str(d), "lm_head.weight", rows[:-1]) != k_rows
    wq, bs, _ = nd.build_or_load(str(d), "lm_head.weight", rows, device="cpu",
                                 cache_dir=str(cache))
    ewq, ebs, _ = _expected(head[rows])
    assert np.array_equal(wq.numpy(), ewq) and np.array_equal(bs.numpy(), ebs)
    shard = d / "model-00002-of-00002.safetensors"
    st = os.stat(shard)
    os.utime(shard, (st.st_atime, st.st_mtime + 10))  # a rewritten checkpoint
    assert nd.cache_key(str(d), "lm_head.weight", rows) != k_rows


def test_missing_tensor(model_dir):
    d, _ = model_dir
    with pytest.raises(FileNotFoundError):
        nd.find_shard(str(d), "no.such.weight")

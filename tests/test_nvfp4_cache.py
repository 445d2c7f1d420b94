"""Load-time NVFP4 packing with its on-disk cache (nvfp4_dense.py), on the CPU: the shard
lookup (index json or safetensors headers), row-subset reads, the cache key (changes with
the row list, the shard's identity and the packing format), reuse of a valid cached pack,
repacking when the cached file's metadata does not match, and no partial file left behind.
The packer is injected: the oracle's quantiser stands in for the GPU kernel here (the GPU
kernel is pinned to the same codes in tests/test_gpu_nvfp4.py)."""

import json
import os

import numpy as np
import pytest
import torch

from flash_next_rtxpro6000_b200 import nvfp4_dense as nd
from oracle import nvfp4 as onv


def _oracle_pack(w):
    wq, bs, gs = onv.quantize(w.float().numpy())
    return (torch.from_numpy(wq), torch.from_numpy(bs),
            torch.from_numpy(np.asarray(gs, np.float32).reshape(1)))


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


@pytest.mark.parametrize("with_index", [False, True])
def test_pack_cache_and_reuse(model_dir, tmp_path, monkeypatch, with_index):
    d, head = model_dir
    if with_index:
        (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {
            "lm_head.weight": "model-00002-of-00002.safetensors",
            "model.norm.weight": "model-00001-of-00002.safetensors"}}))
    assert nd.find_shard(str(d), "lm_head.weight").endswith("model-00002-of-00002.safetensors")
    cache = tmp_path / "cache"
    wq, bs, gs = nd.build_or_load(str(d), "lm_head.weight", device="cpu", cache_dir=str(cache),
                                  pack=_oracle_pack)
    ewq, ebs, egs = _oracle_pack(head)
    assert torch.equal(wq, ewq) and torch.equal(bs, ebs) and torch.equal(gs, egs)
    files = os.listdir(cache)
    assert len(files) == 1 and files[0].endswith(".nvfp4.safetensors") and "partial" not in files[0]

    def no_read(*a, **k):
        raise AssertionError("the cached pack must be reused")

    monkeypatch.setattr(nd, "read_rows", no_read)
    wq2, bs2, gs2 = nd.build_or_load(str(d), "lm_head.weight", device="cpu", cache_dir=str(cache),
                                     pack=_oracle_pack)
    assert torch.equal(wq2, wq) and torch.equal(bs2, bs) and torch.equal(gs2, gs)


def test_row_subset_reads_and_key_changes(model_dir, tmp_path, monkeypatch):
    d, head = model_dir
    rows = torch.tensor([5, 0, 77, 31, 90, 2, 64, 13, 14, 15, 5], dtype=torch.int64)
    assert torch.equal(nd.read_rows(str(d), "lm_head.weight", rows), head[rows])
    cache = tmp_path / "cache"
    k_all = nd.cache_key(str(d), "lm_head.weight", None)
    k_rows = nd.cache_key(str(d), "lm_head.weight", rows)
    assert k_all != k_rows
    assert nd.cache_key(str(d), "lm_head.weight", rows[:-1]) != k_rows
    wq, bs, _ = nd.build_or_load(str(d), "lm_head.weight", rows, device="cpu",
                                 cache_dir=str(cache), pack=_oracle_pack)
    ewq, ebs, _ = _oracle_pack(head[rows])
    assert torch.equal(wq, ewq) and torch.equal(bs, ebs)
    shard = d / "model-00002-of-00002.safetensors"
    st = os.stat(shard)
    os.utime(shard, (st.st_atime, st.st_mtime + 10))  # a rewritten checkpoint
    assert nd.cache_key(str(d), "lm_head.weight", rows) != k_rows
    monkeypatch.setattr(nd, "PACK_FORMAT", nd.PACK_FORMAT + "-next")  # a new packing version
    assert nd.cache_key(str(d), "lm_head.weight", None) != k_all


def test_mismatched_cache_file_is_repacked(model_dir, tmp_path):
    from safetensors.torch import save_file

    d, head = model_dir
    cache = tmp_path / "cache"
    key = nd.cache_key(str(d), "lm_head.weight", None)
    path = nd._cache_path(str(cache), "lm_head.weight", key)
    os.makedirs(cache)
    # a file under the right name whose content is another format / shape
    save_file({"wq": torch.zeros(4, 4, dtype=torch.uint8), "bs": torch.zeros(4, 1, dtype=torch.uint8),
               "gscale": torch.ones(1)}, path,
              metadata={"format": "something-else", "key": key, "rows": "4", "cols": "8"})
    wq, bs, gs = nd.build_or_load(str(d), "lm_head.weight", device="cpu", cache_dir=str(cache),
                                  pack=_oracle_pack)
    ewq, ebs, egs = _oracle_pack(head)
    assert torch.equal(wq, ewq) and torch.equal(bs, ebs) and torch.equal(gs, egs)
    from safetensors import safe_open

    with safe_open(path, framework="pt") as fh:  # replaced by a valid pack
        assert fh.metadata()["format"] == nd.PACK_FORMAT


def test_missing_tensor(model_dir):
    d, _ = model_dir
    with pytest.raises(FileNotFoundError):
        nd.find_shard(str(d), "no.such.weight")

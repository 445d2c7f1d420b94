"""NVFP4 dense lm_head: load-time packing of the checkpoint's rows with an on-disk cache,
and the linear method that serves the packed head through ``w4a16_nvfp4_gemv``.

Counterpart of the reference's NVFP4 dense path (python/sglang/srt/layers/quantization/
nvfp4_dense.py, added by patches/sglang/series/0095-N1-stage-A-integration-SGLANG_MTP_
LMHEAD_NVFP4-1.patch; the target head wiring in 0096-...patch:83-120).  What a caller
relies on is kept: ``build_or_load(model_dir, tensor_name, rows)`` returns the packed
(wq, bs, gscale) of the checkpoint's own rows (never of an already quantised copy: two
lossy steps in a row cost argmax agreement), and ``NVFP4DenseLinearMethod`` offers the
logits processor's ``apply`` / ``apply_into`` (None declines) on a layer prepared by
``attach``.

The cache is this library's own format: a safetensors file holding wq, bs and gscale,
whose metadata records the packing format, the shapes and the source.  Its name carries
a key over everything the packed bytes depend on (the packing format, the model
directory, the tensor, its shard's name / size / mtime and the exact row list), so a
changed checkpoint, row set or packing version never loads a stale file; a file whose
metadata does not match what the key promises is repacked.  Files are written under a
temporary name and renamed into place, so concurrent loaders see the whole file or none.
Packing runs the library's quantise kernel on the GPU (``quantize_nvfp4``).
"""

from __future__ import annotations

import hashlib
import json
import logging
import os
import struct
import time
from typing import Callable, Dict, List, Optional, Tuple

import torch

from .w4a16_nvfp4_gemv import dequantize_nvfp4, quantize_nvfp4, w4a16_nvfp4_gemv

logger = logging.getLogger(__name__)

#: Version of the packed layout and quantiser; part of every cache key and file.
PACK_FORMAT = "fnx-nvfp4/e2m1-lo-nibble-even-k/e4m3-block16/fp32-global/v1"

#: Where packed heads are cached (FNX_NVFP4_CACHE_DIR, else ~/.cache/fnx/nvfp4).
CACHE_DIR = os.environ.get("FNX_NVFP4_CACHE_DIR") or os.path.join(
    os.path.expanduser("~"), ".cache", "fnx", "nvfp4")

#: Head rows dequantised per GEMM by the wide-M path (bounds the bf16 transient).
WIDE_M_ROW_CHUNK = 16384

Packed = Tuple[torch.Tensor, torch.Tensor, torch.Tensor]


# ---------------------------------------------------------------------- checkpoint access
def _safetensors_names(path: str) -> List[str]:
    """Tensor names in a safetensors file, from its JSON header alone."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    return [k for k in header if k != "__metadata__"]


def find_shard(model_dir: str, tensor_name: str) -> str:
    """The safetensors file under ``model_dir`` that stores ``tensor_name``: the one the
    index json names, or the first whose header lists it."""
    for index in ("model.safetensors.index.json",):
        p = os.path.join(model_dir, index)
        if os.path.isfile(p):
            with open(p) as f:
                shard = json.load(f).get("weight_map", {}).get(tensor_name)
            if shard:
                return os.path.join(model_dir, shard)
    shards = sorted(n for n in os.listdir(model_dir) if n.endswith(".safetensors"))
    for name in shards:
        path = os.path.join(model_dir, name)
        if tensor_name in _safetensors_names(path):
            return path
    raise FileNotFoundError(f"no safetensors file under {model_dir} holds {tensor_name!r}")


def _row_list(rows: Optional[torch.Tensor]) -> Optional[List[int]]:
    return None if rows is None else rows.detach().to("cpu", torch.int64).reshape(-1).tolist()


def read_rows(model_dir: str, tensor_name: str, rows: Optional[torch.Tensor] = None
              ) -> torch.Tensor:
    """``tensor_name`` as stored in the checkpoint, or only ``rows`` of it (in that order).
    Each maximal run of consecutive requested rows is one slice read."""
    from safetensors import safe_open

    path = find_shard(model_dir, tensor_name)
    with safe_open(path, framework="pt", device="cpu") as fh:
        want = _row_list(rows)
        if want is None:
            return fh.get_tensor(tensor_name)
        sl = fh.get_slice(tensor_name)
        order = sorted(set(want))
        pieces: Dict[int, torch.Tensor] = {}
        i = 0
        while i < len(order):
            j = i
            while j + 1 < len(order) and order[j + 1] == order[j] + 1:
                j += 1
            block = sl[order[i]:order[j] + 1]
            for r in range(order[i], order[j] + 1):
                pieces[r] = block[r - order[i]]
            i = j + 1
        return torch.stack([pieces[r] for r in want])


# ---------------------------------------------------------------------- cache
def cache_key(model_dir: str, tensor_name: str, rows: Optional[torch.Tensor]) -> str:
    """Hex key over what the packed bytes depend on: packing format, model directory,
    tensor, its shard's identity (name, size, mtime) and the row list."""
    shard = find_shard(model_dir, tensor_name)
    st = os.stat(shard)
    want = _row_list(rows)
    row_id = "all" if want is None else hashlib.sha256(
        torch.tensor(want, dtype=torch.int64).numpy().tobytes()).hexdigest()
    desc = {"format": PACK_FORMAT, "model": os.path.realpath(model_dir), "tensor": tensor_name,
            "shard": [os.path.basename(shard), st.st_size, st.st_mtime_ns],
            "rows": [len(want), row_id] if want is not None else "all"}
    return hashlib.sha256(json.dumps(desc, sort_keys=True).encode()).hexdigest()[:40]


def _cache_path(cache_dir: str, tensor_name: str, key: str) -> str:
    safe = "".join(ch if ch.isalnum() or ch in "._-" else "_" for ch in tensor_name)
    return os.path.join(cache_dir, f"{safe}.{key}.nvfp4.safetensors")


def _load_cached(path: str, key: str, device) -> Optional[Packed]:
    from safetensors import safe_open

    try:
        with safe_open(path, framework="pt", device="cpu") as fh:
            meta = fh.metadata() or {}
            t = {k: fh.get_tensor(k) for k in ("wq", "bs", "gscale")}
    except Exception as e:  # unreadable or partial: repack
        logger.warning("NVFP4 cache %s unreadable (%s); repacking", os.path.basename(path), e)
        return None
    n, k = int(meta.get("rows", -1)), int(meta.get("cols", -1))
    ok = (meta.get("format") == PACK_FORMAT and meta.get("key") == key and n > 0 and k > 0
          and t["wq"].dtype == torch.uint8 and tuple(t["wq"].shape) == (n, k // 2)
          and t["bs"].dtype == torch.uint8 and tuple(t["bs"].shape) == (n, k // 16)
          and t["gscale"].dtype == torch.float32 and t["gscale"].numel() == 1)
    if not ok:
        logger.warning("NVFP4 cache %s does not match its key or format; repacking",
                       os.path.basename(path))
        return None
    return t["wq"].to(device), t["bs"].to(device), t["gscale"].reshape(1).to(device)


def _store(path: str, key: str, packed: Packed, source: str) -> None:
    from safetensors.torch import save_file

    wq, bs, gs = (t.detach().to("cpu").contiguous() for t in packed)
    meta = {"format": PACK_FORMAT, "key": key, "rows": str(wq.shape[0]),
            "cols": str(wq.shape[1] * 2), "source": source}
    tmp = f"{path}.{os.getpid()}.partial"
    save_file({"wq": wq, "bs": bs, "gscale": gs.reshape(1)}, tmp, metadata=meta)
    os.replace(tmp, path)  # atomic on one file system


def build_or_load(model_dir: str, tensor_name: str, rows: Optional[torch.Tensor] = None,
                  device="cuda", label: str = "", cache_dir: Optional[str] = None,
                  pack: Optional[Callable[[torch.Tensor], Packed]] = None) -> Packed:
    """(wq [N, K/2] uint8, bs [N, K/16] uint8 e4m3, gscale [1] fp32) on ``device`` for the
    checkpoint tensor (or its ``rows``): from the cache when a valid file for this key
    exists, else packed now and cached.  ``pack`` replaces the GPU quantiser (the rows
    are handed to it on ``device``)."""
    cache_dir = cache_dir or CACHE_DIR
    key = cache_key(model_dir, tensor_name, rows)
    path = _cache_path(cache_dir, tensor_name, key)
    name = label or tensor_name
    if os.path.isfile(path):
        t0 = time.perf_counter()
        hit = _load_cached(path, key, device)
        if hit is not None:
            logger.info("NVFP4 %s: cached pack loaded in %.2f s", name, time.perf_counter() - t0)
            return hit
    t0 = time.perf_counter()
    src = read_rows(model_dir, tensor_name, rows).to(device)
    packed = (pack or quantize_nvfp4)(src)
    del src
    os.makedirs(cache_dir, exist_ok=True)
    _store(path, key, packed, f"{os.path.realpath(model_dir)}:{tensor_name}")
    logger.info("NVFP4 %s: packed %d x %d in %.2f s", name, packed[0].shape[0],
                packed[0].shape[1] * 2, time.perf_counter() - t0)
    return packed


# ---------------------------------------------------------------------- linear method
class NVFP4DenseLinearMethod:
    """Weight-only NVFP4 linear method for an lm_head (the quant-method hook the logits
    processor calls).  ``attach`` puts the packed tensors on the layer (``nvfp4_wq``,
    ``nvfp4_bs``, ``nvfp4_gscale``; ``layer.weight`` points at the codes, since dispatch
    only checks that a weight exists), so one instance serves any number of layers."""

    #: widest call served by the GEMV; wider calls (prefill, extend) take the GEMM path
    MAX_GEMV_TOKENS = 16

    def __init__(self, name: str = "lm_head"):
        self.name = name

    @staticmethod
    def attach(layer, wq: torch.Tensor, bs: torch.Tensor, gscale: torch.Tensor) -> None:
        layer.nvfp4_wq, layer.nvfp4_bs, layer.nvfp4_gscale = wq, bs, gscale
        layer.weight = wq

    @classmethod
    def _packed(cls, layer) -> Optional[Packed]:
        wq = getattr(layer, "nvfp4_wq", None)
        return None if wq is None else (wq, layer.nvfp4_bs, layer.nvfp4_gscale)

    @classmethod
    def _serves(cls, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dim() == 2 and x.dtype == torch.bfloat16 and x.stride(1) == 1
                and 1 <= x.shape[0] <= cls.MAX_GEMV_TOKENS)

    def apply(self, layer, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Logits [M, N] (bf16) of x [M, K]."""
        p = self._packed(layer)
        if p is None:
            raise RuntimeError(f"{self.name}: no packed NVFP4 weight attached")
        y = w4a16_nvfp4_gemv(x, *p) if self._serves(x) else self._gemm(p, x)
        return y if bias is None else y + bias

    def apply_into(self, layer, x: torch.Tensor, out: torch.Tensor,
                   bias: Optional[torch.Tensor] = None):
        """Logits written into ``out`` ([M, N] bf16, or the fp32 next-token buffer holding
        bf16 values) by the GEMV; None declines (bias, too wide, no packed weight, a
        destination of another shape or type), leaving the caller's own path."""
        p = self._packed(layer)
        if p is None or bias is not None or not self._serves(x):
            return None
        shape_ok = tuple(out.shape) == (x.shape[0], p[0].shape[0]) and out.stride(1) == 1
        if not shape_ok or out.dtype not in (torch.bfloat16, torch.float32) or out.device != x.device:
            return None
        return w4a16_nvfp4_gemv(x, *p, out=out)

    @staticmethod
    def _gemm(p: Packed, x: torch.Tensor) -> torch.Tensor:
        """Many tokens: bf16 GEMMs over the head dequantised WIDE_M_ROW_CHUNK rows at a
        time (one bf16 slab, reused), so the head is read once, not once per 16 tokens."""
        wq, bs, gs = p
        N, K = wq.shape[0], wq.shape[1] * 2
        xb = x.to(torch.bfloat16)
        y = torch.empty((x.shape[0], N), dtype=torch.bfloat16, device=x.device)
        slab = torch.empty((min(N, WIDE_M_ROW_CHUNK), K), dtype=torch.bfloat16, device=x.device)
        per_row = gs.numel() > 1
        for r0 in range(0, N, WIDE_M_ROW_CHUNK):
            r1 = min(N, r0 + WIDE_M_ROW_CHUNK)
            w = dequantize_nvfp4(wq[r0:r1], bs[r0:r1], gs[r0:r1] if per_row else gs,
                                 dtype=torch.bfloat16, out=slab[:r1 - r0])
            torch.mm(xb, w.t(), out=y[:, r0:r1])
        return y

"""NVFP4 dense lm_head: load-time packing with an on-disk cache, and the linear method
that serves it through ``w4a16_nvfp4_gemv`` (the reference's
python/sglang/srt/layers/quantization/nvfp4_dense.py, patches/sglang/series/
0095-N1-stage-A-integration-SGLANG_MTP_LMHEAD_NVFP4-1.patch:90-260, used for the
target head by 0096-…patch:83-120).

* The rows are packed from the checkpoint's own (bf16) tensor, read lazily from its
  safetensors shard, never from an already-quantised copy: two lossy steps in a row cost
  argmax agreement.
* Packing is deterministic, so the result is cached under a key over the model
  directory, the tensor name, the shard's name / size / mtime and the exact row set
  (a hot-vocabulary map); the file is written under a temporary name and moved into
  place with ``os.replace``, so two processes starting together never read half a file.
* ``NVFP4DenseLinearMethod`` provides what the logits processor needs of a quant method:
  ``apply`` (logits) and ``apply_into`` (into the shared fp32 next-token buffer, None to
  decline); calls wider than the GEMV's 16 tokens dequantise the weight in row chunks
  and run a GEMM.
"""

from __future__ import annotations

import hashlib
import json
import logging
import os
import time
from typing import Optional

import torch

from .w4a16_nvfp4_gemv import dequantize_nvfp4, quantize_nvfp4, w4a16_nvfp4_gemv

logger = logging.getLogger(__name__)

#: Where packed weights are cached: FNX_NVFP4_CACHE_DIR, else the reference's
#: SGLANG_NVFP4_CACHE_DIR, else ~/.cache/fnx/nvfp4.
CACHE_DIR = (os.environ.get("FNX_NVFP4_CACHE_DIR") or os.environ.get("SGLANG_NVFP4_CACHE_DIR")
             or os.path.join(os.path.expanduser("~/.cache/fnx"), "nvfp4"))

#: Rows dequantised at a time by the wide-M path (bounds its transient).
WIDE_M_ROW_CHUNK = 16384


def _index_file(model_dir: str) -> Optional[str]:
    for name in ("model.safetensors.index.json", "pytorch_model.bin.index.json"):
        p = os.path.join(model_dir, name)
        if os.path.exists(p):
            return p
    return None


def find_shard(model_dir: str, tensor_name: str) -> str:
    """Path of the safetensors shard that holds ``tensor_name``: from the index json when
    there is one, else by reading each shard's header."""
    idx = _index_file(model_dir)
    if idx is not None:
        with open(idx) as f:
            where = json.load(f).get("weight_map", {}).get(tensor_name)
        if where is not None:
            return os.path.join(model_dir, where)
    from safetensors import safe_open

    for name in sorted(os.listdir(model_dir)):
        if not name.endswith(".safetensors"):
            continue
        path = os.path.join(model_dir, name)
        with safe_open(path, framework="pt", device="cpu") as fh:
            if tensor_name in fh.keys():
                return path
    raise FileNotFoundError(f"{tensor_name} is in no shard under {model_dir}")


def _shard_identity(path: str) -> str:
    st = os.stat(path)
    return f"{os.path.basename(path)}:{st.st_size}:{int(st.st_mtime)}"


def _row_set(rows: Optional[torch.Tensor]) -> str:
    if rows is None:
        return "all"
    r = rows.detach().to("cpu", torch.int64).contiguous()
    return f"{r.numel()}-{hashlib.sha256(r.numpy().tobytes()).hexdigest()[:16]}"


def cache_key(model_dir: str, tensor_name: str, rows: Optional[torch.Tensor]) -> str:
    """32 hex digits of sha256 over everything the packed bytes depend on."""
    parts = (os.path.realpath(model_dir), tensor_name,
             _shard_identity(find_shard(model_dir, tensor_name)), _row_set(rows))
    return hashlib.sha256("|".join(parts).encode()).hexdigest()[:32]


def read_rows(model_dir: str, tensor_name: str, rows: Optional[torch.Tensor] = None
              ) -> torch.Tensor:
    """The tensor's rows as stored in the checkpoint (all of them, or ``rows`` in that
    order); only the requested rows are read from disk."""
    from safetensors import safe_open

    with safe_open(find_shard(model_dir, tensor_name), framework="pt", device="cpu") as fh:
        if rows is None:
            return fh.get_tensor(tensor_name)
        sl = fh.get_slice(tensor_name)
        return torch.cat([sl[i:i + 1, :] for i in rows.detach().to("cpu", torch.int64).tolist()])


def build_or_load(model_dir: str, tensor_name: str, rows: Optional[torch.Tensor] = None,
                  device="cuda", label: str = "", cache_dir: Optional[str] = None):
    """-> (wq [N, K/2] uint8, bs [N, K/16] uint8 e4m3, gscale [1] fp32) on ``device``,
    from the cache when it holds this exact tensor and row set, else packed and cached."""
    cache_dir = cache_dir or CACHE_DIR
    key = cache_key(model_dir, tensor_name, rows)
    path = os.path.join(cache_dir, f"{tensor_name.replace('/', '_')}.{key}.pt")
    tag = label or tensor_name
    if os.path.exists(path):
        t0 = time.time()
        blob = torch.load(path, map_location=device, weights_only=True)
        logger.info("NVFP4 %s: packed weight from the cache in %.2fs (%s)", tag,
                    time.time() - t0, os.path.basename(path))
        return blob["wq"], blob["bs"], blob["gscale"]
    t0 = time.time()
    w = read_rows(model_dir, tensor_name, rows)
    wq, bs, gscale = quantize_nvfp4(w.to(device))
    del w
    os.makedirs(cache_dir, exist_ok=True)
    tmp = f"{path}.tmp{os.getpid()}"
    torch.save({"wq": wq.cpu(), "bs": bs.cpu(), "gscale": gscale.cpu()}, tmp)
    os.replace(tmp, path)  # readers see either no file or the whole file
    logger.info("NVFP4 %s: packed %s in %.2fs -> %s", tag, tuple(wq.shape), time.time() - t0,
                os.path.basename(path))
    return wq, bs, gscale


class NVFP4DenseLinearMethod:
    """Weight-only NVFP4 for an lm_head.  The packed tensors live on the layer
    (``nvfp4_wq``, ``nvfp4_bs``, ``nvfp4_gscale``), so one instance serves several layers;
    ``layer.weight`` is set to the codes because the dispatch only checks that it exists."""

    def __init__(self, name: str = "lm_head"):
        self.name = name

    @staticmethod
    def attach(layer, wq, bs, gscale) -> None:
        layer.nvfp4_wq = wq
        layer.nvfp4_bs = bs
        layer.nvfp4_gscale = gscale
        layer.weight = wq

    @staticmethod
    def _gemv_ok(layer, x: torch.Tensor) -> bool:
        return (getattr(layer, "nvfp4_wq", None) is not None and x.dim() == 2
                and x.shape[0] <= 16 and x.dtype == torch.bfloat16 and x.is_cuda
                and x.stride(1) == 1)

    def apply(self, layer, x: torch.Tensor, bias: Optional[torch.Tensor] = None):
        if self._gemv_ok(layer, x):
            y = w4a16_nvfp4_gemv(x, layer.nvfp4_wq, layer.nvfp4_bs, layer.nvfp4_gscale)
        else:
            y = self._wide_m(layer, x)
        return y if bias is None else y + bias

    def apply_into(self, layer, x: torch.Tensor, out: torch.Tensor,
                   bias: Optional[torch.Tensor] = None):
        """Logits into ``out`` (bf16 or the shared fp32 buffer) through the GEMV, or None
        when this call is not one it serves."""
        if bias is not None or not self._gemv_ok(layer, x):
            return None
        N = layer.nvfp4_wq.shape[0]
        if (tuple(out.shape) != (x.shape[0], N) or out.dtype not in (torch.bfloat16, torch.float32)
                or out.device != x.device or out.stride(1) != 1):
            return None
        return w4a16_nvfp4_gemv(x, layer.nvfp4_wq, layer.nvfp4_bs, layer.nvfp4_gscale, out=out)

    @staticmethod
    def _wide_m(layer, x: torch.Tensor) -> torch.Tensor:
        """More tokens than the GEMV takes (prefill / extend): a GEMM on the weight
        dequantised WIDE_M_ROW_CHUNK rows at a time, so the bf16 copy never exists whole
        (re-running the GEMV per 16 tokens would re-stream the whole weight each time)."""
        wq, bs, gs = layer.nvfp4_wq, layer.nvfp4_bs, layer.nvfp4_gscale
        N = wq.shape[0]
        y = torch.empty((x.shape[0], N), dtype=torch.bfloat16, device=x.device)
        for r0 in range(0, N, WIDE_M_ROW_CHUNK):
            r1 = min(N, r0 + WIDE_M_ROW_CHUNK)
            w = dequantize_nvfp4(wq[r0:r1], bs[r0:r1], gs).to(torch.bfloat16)
            torch.mm(x.to(torch.bfloat16), w.t(), out=y[:, r0:r1])
            del w
        return y

"""Multi-GPU forms of the hot path over torch.distributed (NCCL on NVLink / NVSwitch).

One process per GPU.  Two sharding schemes, each with exactly one exchange step:

* vocab-sharded lm_head: rank g holds rows [g*V/G, (g+1)*V/G).  The GEMV writes its
  shard's logits and a 64-bit argmax key per token (bf16 value key << 32 | ~global_row);
  the MAX of the M keys over ranks picks the global greedy token with the lowest row on
  ties, bit-identical to the single-GPU argmax because every rank rounds to bf16 before
  comparing.  ``vocab_sharded_lm_head`` does that MAX inside the GEMV's last CTA over
  NVLink peer memory (``PeerExchange``, one launch per rank, no NCCL);
  ``sharded_lm_head_argmax`` does it with an NCCL MAX all-reduce.  ``all_gather_logits``
  optionally assembles the full [M, V] logits.
* expert-sharded MoE (``expert_sharded_moe``): rank g holds experts
  [g*E/G, (g+1)*E/G) (and rank 0 the shared expert).  Each rank computes the fp32 partial
  sum of its experts' routes; a SUM all-reduce of the [M, H] partials and one rounding to
  bf16 give the layer output.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib, errors
from ._lib import check, ptr
from .draft_moe_gemv import DraftMoeWorkspace, SharedExpert, draft_moe_gemv
from .w8a16_gemv import PDL, _activation, _scale_kind, _stream, _weight_kind, _workspace


def shard_rows(V: int, world: int, rank: int):
    """(first row, rows) of this rank's vocab shard."""
    if V % world:
        raise ValueError(f"vocab {V} is not divisible by {world} ranks")
    n = V // world
    return rank * n, n


def lm_head_keys(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, row_offset: int,
                 out: Optional[torch.Tensor] = None, keys: Optional[torch.Tensor] = None,
                 pdl: Optional[bool] = None):
    """Local shard GEMV + the shard's argmax keys (int64 [M], global row ids)."""
    M, K = x.shape
    N = w.shape[0]
    x = _activation(x)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device) if out is None else out
    k = torch.empty(M, dtype=torch.int64, device=x.device) if keys is None else keys
    s, skind = _scale_kind(scale, N)
    ws = _workspace(x.device)
    rc = _lib.lib().fnx_w8a16_gemv(
        ptr(x), x.stride(0), ptr(w), w.stride(0) * w.element_size(), _weight_kind(w), ptr(s),
        skind, ptr(y), y.stride(0), None, 0, 0, int(y.dtype == torch.float32), None, ptr(k),
        row_offset, M, N, K, None, ctypes.byref(ws.c), int(PDL if pdl is None else pdl),
        _stream(x))
    check(rc, "lm_head_keys")
    return y, k


def decode_keys(keys: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    M = keys.numel()
    o = torch.empty(M, dtype=torch.int64, device=keys.device) if out is None else out
    check(_lib.lib().fnx_argmax_decode(ptr(keys), ptr(o), M, _stream(keys)), "argmax_decode")
    return o


def sharded_lm_head_argmax(x, w_shard, s_shard, row_offset: int, out=None, argmax_out=None,
                           group=None, pdl: Optional[bool] = True):
    """Greedy token of a vocab-sharded head: local GEMV, MAX all-reduce of the keys."""
    y, keys = lm_head_keys(x, w_shard, s_shard, row_offset, out=out, pdl=pdl)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    return y, decode_keys(keys, argmax_out)


class PeerExchange:
    """Buffers of the in-kernel greedy-key exchange (fnx_w8a16_gemv_vocab_sharded): one
    small device buffer per rank, mapped into every other rank's process by CUDA IPC.
    Collective over ``group`` (every rank constructs it together); ``close`` likewise.
    Without an initialised process group it is the one-rank exchange (with itself)."""

    def __init__(self, device=None, group=None):
        self.group = group
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        multi = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if multi else 1
        self.rank = dist.get_rank(group) if multi else 0
        if self.world > _lib.MAX_PEERS:
            raise NotImplementedError(f"at most {_lib.MAX_PEERS} ranks")
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            buf = ctypes.c_void_p()
            check(lib.fnx_peer_alloc(ctypes.byref(buf)), "fnx_peer_alloc")
            self.buf = buf.value
            handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
            check(lib.fnx_ipc_get_handle(self.buf, handle), "fnx_ipc_get_handle")
            handles = [None] * self.world
            if multi:
                dist.all_gather_object(handles, handle.raw, group=group)
            else:
                handles[0] = handle.raw
            self.opened = []
            bufs = (ctypes.c_void_p * self.world)()
            for r, h in enumerate(handles):
                if r == self.rank:
                    bufs[r] = self.buf
                    continue
                p = ctypes.c_void_p()
                check(lib.fnx_ipc_open(ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES),
                                       ctypes.byref(p)), "fnx_ipc_open")
                bufs[r] = p.value
                self.opened.append(p.value)
            check(lib.fnx_peer_setup(self.buf, bufs, self.world, self.rank), "fnx_peer_setup")
        if multi:
            dist.barrier(group=group)

    def set_wait_limit(self, seconds: float) -> None:
        """Limit of each call's wait for the other ranks' keys (default 2 s)."""
        check(_lib.lib().fnx_peer_set_wait_limit(self.buf, int(seconds * 1e9)),
              "fnx_peer_set_wait_limit")

    def close(self):
        """Unmap the other ranks' buffers and free this rank's (after every rank's last
        call has finished)."""
        if self.buf is None:
            return
        torch.cuda.synchronize(self.device)
        if dist.is_available() and dist.is_initialized():
            dist.barrier(group=self.group)
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self.opened:
                check(lib.fnx_ipc_close(p), "fnx_ipc_close")
            check(lib.fnx_peer_free(self.buf), "fnx_peer_free")
        self.opened, self.buf = [], None


def vocab_sharded_lm_head(x, w_shard, s_shard, row_offset: int, exchange: PeerExchange,
                          out=None, argmax_out=None, pdl: Optional[bool] = True,
                          check_errors: bool = False):
    """Greedy token of a vocab-sharded head in one launch per rank: the shard's GEMV with
    the MAX over ranks of the greedy keys done by its last CTA over NVLink (no NCCL).

    If another rank does not publish its key within the exchange's wait limit (2 s by
    default, ``PeerExchange.set_wait_limit``), or is two or more calls ahead, this rank
    keeps its own shard's token and the GEMV scratch's error flag is set: ``argmax_out``
    is then not the global greedy token.  ``check_errors=True`` synchronises the stream after the
    call, clears the flag and raises ``errors.DeviceWaitError`` when it was set (outside
    graph capture only); otherwise ``errors.check_device_errors()`` reports it later."""
    M, K = x.shape
    N = w_shard.shape[0]
    x = _activation(x)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device) if out is None else out
    am = torch.empty(M, dtype=torch.int64, device=x.device) if argmax_out is None else argmax_out
    s, skind = _scale_kind(s_shard, N)
    ws = _workspace(x.device)
    rc = _lib.lib().fnx_w8a16_gemv_vocab_sharded(
        ptr(x), x.stride(0), ptr(w_shard), w_shard.stride(0) * w_shard.element_size(),
        _weight_kind(w_shard), ptr(s), skind, ptr(y), y.stride(0), int(y.dtype == torch.float32),
        ptr(am), row_offset, M, N, K, exchange.buf, None, ctypes.byref(ws.c),
        int(PDL if pdl is None else pdl), _stream(x))
    check(rc, "vocab_sharded_lm_head")
    if check_errors:
        errors.check_flag(ws.error_flag, "vocab_sharded_lm_head")
    return y, am


def all_gather_logits(local: torch.Tensor, group=None) -> torch.Tensor:
    """[M, V/G] per rank -> [M, V] (row-major by rank)."""
    world = dist.get_world_size(group)
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def expert_sharded_moe(*, hidden_states, topk_ids, topk_weights, w13_weight,
                       w13_blockscale_swizzled, w13_weight_scale_2, w2_weight,
                       w2_blockscale_swizzled, w2_weight_scale_2, expert_offset: int,
                       workspace: DraftMoeWorkspace, shared_expert: Optional[SharedExpert] = None,
                       group=None, partial: Optional[torch.Tensor] = None) -> torch.Tensor:
    """MoE layer with this rank's expert slice; SUM all-reduce of fp32 partials."""
    part = draft_moe_gemv(
        hidden_states=hidden_states, topk_ids=topk_ids, topk_weights=topk_weights,
        w13_weight=w13_weight, w13_blockscale_swizzled=w13_blockscale_swizzled,
        w13_weight_scale_2=w13_weight_scale_2, w2_weight=w2_weight,
        w2_blockscale_swizzled=w2_blockscale_swizzled, w2_weight_scale_2=w2_weight_scale_2,
        workspace=workspace, shared_expert=shared_expert, expert_offset=expert_offset,
        out=partial, out_f32=True)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return part.to(torch.bfloat16)


# ------------------------------------------------------------------------------------
# Host form of the argmax key (the device builds the same 64-bit key per row).
# ------------------------------------------------------------------------------------
def order_key16(bf16_bits: int) -> int:
    """Order-preserving key of a bf16 bit pattern; -0 folds onto +0."""
    b = bf16_bits & 0xFFFF
    if b == 0x8000:
        b = 0
    return (~b & 0xFFFF) if b & 0x8000 else (b | 0x8000)


def encode_key(bf16_bits: int, row: int) -> int:
    return (order_key16(bf16_bits) << 32) | (0xFFFFFFFF - row)


def decode_key(key: int) -> int:
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)

"""Host-side logic that needs no GPU: destination validation (w8a16_gemv.py:599-639),
scratch slots, MoE shape gating (0112-...patch:289-305), argmax key encoding, the
synthetic generators' byte model, and the multi-rank exchange of the sharded head and
the expert-sharded MoE on 2 gloo ranks."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import importlib

from flash_next_rtxpro6000_b200 import sharded, synthetic
from oracle import numerics

# the package re-exports functions under the module names; take the modules themselves
dmg = importlib.import_module("flash_next_rtxpro6000_b200.draft_moe_gemv")
w8 = importlib.import_module("flash_next_rtxpro6000_b200.w8a16_gemv")


def test_out_validation():
    d = torch.device("cpu")
    assert w8._out_or_new(None, 2, 8, d).shape == (2, 8)
    good = torch.empty(2, 8, dtype=torch.float32)
    assert w8._out_or_new(good, 2, 8, d) is good
    for bad in (torch.empty(2, 9), torch.empty(2, 8, dtype=torch.float16), torch.empty(8, 2).t()):
        with pytest.raises(ValueError):
            w8._out_or_new(bad, 2, 8, d)
    with pytest.raises(ValueError):
        w8._split_dests(None, torch.empty(2, 3), 0, 2, 8, d)
    y, y2, s = w8._split_dests(None, None, 0, 2, 8, d)
    assert y2 is None and s == 0


def test_scratch_slot_nesting():
    assert w8._SLOT == 0
    with w8.scratch_slot(1):
        assert w8._SLOT == 1
        with w8.scratch_slot(0):
            assert w8._SLOT == 0
        assert w8._SLOT == 1
    assert w8._SLOT == 0


def test_unsupported_reason():
    assert dmg.unsupported_reason(hidden_size=2048, intermediate_size=512) is None
    assert dmg.unsupported_reason(hidden_size=2560, intermediate_size=640) is None
    assert "multiples of 128" in dmg.unsupported_reason(hidden_size=2000, intermediate_size=512)
    assert dmg.unsupported_reason(hidden_size=8192, intermediate_size=512) is not None


def test_argmax_key_orders_like_torch_argmax():
    rng = np.random.default_rng(0)
    v = numerics.bf16_round(rng.standard_normal(4000).astype(np.float32) * 4)
    v[[10, 200, 3000]] = v.max()  # ties: lowest row must win
    v[5] = -0.0
    bits = numerics.bf16_bits(v)
    keys = [sharded.encode_key(int(b), i) for i, b in enumerate(bits)]
    assert sharded.decode_key(max(keys)) == int(np.argmax(v)) == 10
    zero = [sharded.encode_key(0x8000, 0), sharded.encode_key(0x0000, 1)]
    assert sharded.decode_key(max(zero)) == 0  # -0 == +0 ties -> lowest row


def test_byte_model_matches_survey_figures():
    assert synthetic.w8_head_bytes(151936, 2048, 1, argmax=False) == 311_776_768
    assert synthetic.w8_head_bytes(49152, 2048, 1, argmax=False) == 100_864_000
    assert synthetic.nvfp4_bytes(4096, 2048, 1) == 4_730_880
    assert synthetic.moe_bytes(10, M=1) == 19_472_384


def test_routing_generator():
    ids, w = synthetic.routing(16, seed=0)
    assert ids.shape == (16, 10) and ids.dtype == torch.int32
    assert torch.allclose(w.sum(-1), torch.ones(16))
    for row in ids:
        assert len(set(row.tolist())) == 10


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(1)
        V, M = 4096, 3
        logits = numerics.bf16_round(rng.standard_normal((M, V)).astype(np.float32) * 3)
        logits[1, 17] = logits[1, 3000] = logits[1].max() + 1  # tie across the two shards
        r0, n = sharded.shard_rows(V, world, rank)
        bits = numerics.bf16_bits(logits[:, r0:r0 + n])
        keys = torch.tensor([max(sharded.encode_key(int(b), r0 + j) for j, b in enumerate(row))
                             for row in bits], dtype=torch.int64)
        dist.all_reduce(keys, op=dist.ReduceOp.MAX)
        got = [sharded.decode_key(int(k)) for k in keys]
        # expert-sharded partial sums
        part = torch.full((2, 4), float(rank + 1))
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        q.put((rank, got, np.argmax(logits, axis=-1).tolist(), float(part[0, 0])))
    finally:
        dist.destroy_process_group()


def test_two_rank_exchange_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, want, s in res:
        assert got == want
        assert want[1] == 17
        assert s == 3.0


def test_reference_cfg_tuple_is_ignored():
    """The reference's Triton 7-tuple cfg (w8a16_gemv.py:522-538) maps to the planner."""
    assert w8._cfg((128, 64, 4, False, False, 4, 3)) is None
    assert w8._cfg(None) is None
    assert w8._cfg((8, 4)).warps == 8
    with pytest.raises(ValueError):
        w8._cfg((1, 2, 3, 4, 5, 6))


def test_n_major_weight_is_declined():
    """An N-contiguous [N, K] view (the reference's W_KN case) is declined with
    NotImplementedError before any launch, so a caller keeps its own path."""
    import flash_next_rtxpro6000_b200 as fx

    N, K = 64, 128
    x = torch.zeros(1, K, dtype=torch.bfloat16)
    w = torch.zeros(K, N, dtype=torch.int8).t()  # [N, K], stride (1, N)
    s = torch.ones(N)
    with pytest.raises(NotImplementedError):
        fx.w8a16_gemv(x, w, s)
    with pytest.raises(NotImplementedError):
        fx.w8a16_gemv_silu_mul(x, torch.zeros(K, 2 * N, dtype=torch.int8).t(), torch.ones(2 * N))


def test_device_error_flags_are_read_and_cleared():
    from flash_next_rtxpro6000_b200 import errors

    f1 = torch.zeros(1, dtype=torch.int32)
    f2 = torch.zeros(1, dtype=torch.int32)
    errors.register(f1, "first")
    errors.register(f2, "second")
    errors.check_device_errors(torch.device("cpu"))  # nothing set
    f2.fill_(7)
    with pytest.raises(errors.DeviceWaitError) as ei:
        errors.check_device_errors(torch.device("cpu"))
    assert ei.value.codes == [("second", 7)]
    assert "WAIT_PEER" in str(ei.value)
    assert int(f2.item()) == 0  # cleared
    errors.check_device_errors(torch.device("cpu"))
    f1.fill_(9)
    with pytest.raises(errors.DeviceWaitError):
        errors.check_flag(f1, "first", clear=False)
    assert int(f1.item()) == 9
    f1.zero_()


@pytest.mark.parametrize("H,I", [(2048, 512), (2560, 640), (1024, 256), (2048, 1024)])
def test_fused_moe_ring_stages_are_owned(H, I):
    """The one-launch MoE layer hands ring stages round robin to its producer warps and
    consumer groups and waits on them by phase parity, which is only sound when every
    stage belongs to one producer warp and one consumer group: the stage count must be a
    multiple of both (an odd count faulted on the GPU).  The planner guarantees it for
    every token count, routing width and expert count; a form that does not fit falls back
    to the three-launch layer, which the launch accounting follows."""
    import flash_next_rtxpro6000_b200 as fx

    seen = set()
    for M in range(1, 17):
        for R in (1, 8, 10, 32):
            for E in (1, 64, 256, 512):
                p = fx.moe_plan(M, R, E, H, I)
                if not p["fused"]:
                    assert p["stages"] == 0
                    assert fx.moe_launches_per_call(H, I, num_tokens=M, top_k=R, num_experts=E) == 3
                    continue
                ns, ng = p["stages"], p["groups"]
                assert ng >= 1 and ns >= 4
                assert ns % ng == 0 and ns % 2 == 0, (M, R, E, ns, ng)
                assert 0 < p["smem_bytes"] <= 227 * 1024
                assert fx.moe_launches_per_call(H, I, num_tokens=M, top_k=R, num_experts=E) == 1
                seen.add(ns)
    if (H, I) != (2048, 1024):
        assert seen, "the fused layer is planned for some shape"


def test_dense_path_selector():
    """fnx_set_dense_path switches the dense GEMV form process-wide and reports the
    previous setting; an unknown name is a ValueError (the ABI's FNX_EINVAL)."""
    import flash_next_rtxpro6000_b200 as fx

    prev = fx.set_dense_path("mma")
    try:
        assert fx.set_dense_path("tcgen05") == "mma"
        with fx.dense_path("mma"):
            assert fx.set_dense_path("mma") == "mma"
        assert fx.set_dense_path("auto") == "tcgen05"
        with pytest.raises(ValueError):
            fx.set_dense_path("wgmma")
    finally:
        fx.set_dense_path(prev)


def test_moe_form_selection():
    """The one-token layer serves M = 1 with 256-multiple H and I (I <= 512, H <= 2048);
    every other call, and every call under moe_path("fused"), takes the general
    one-launch layer; an unknown path name is a ValueError (the ABI's FNX_EINVAL)."""
    import flash_next_rtxpro6000_b200 as fx

    assert fx.moe_plan(1, 10, 512, 2048, 512)["form"] == "lean"
    assert fx.moe_kernel_name(2048, 512, True, num_tokens=1) == "moe_lean_kernel"
    assert fx.moe_launches_per_call(2048, 512, num_tokens=1) == 1
    for M, H, I in ((2, 2048, 512), (16, 2048, 512), (1, 2560, 640)):
        assert fx.moe_plan(M, 10, 512, H, I)["form"] == "fused", (M, H, I)
    p = fx.moe_plan(1, 10, 512, 2048, 512)
    assert p["stages"] % p["groups"] == 0 and 0 < p["smem_bytes"] <= 227 * 1024
    with fx.moe_path("fused"):
        assert fx.moe_plan(1, 10, 512, 2048, 512)["form"] == "fused"
    assert fx.moe_plan(1, 10, 512, 2048, 512)["form"] == "lean"
    with pytest.raises(ValueError):
        fx.set_moe_path("lean-ish")

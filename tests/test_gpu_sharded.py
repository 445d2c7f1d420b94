"""Sharded forms on 2 GPUs, against the 1-GPU results: the vocab-sharded lm_head (NCCL
MAX all-reduce of argmax keys, and the exchange inside the GEMV over NVLink peer memory
on three calls in a row) gives the same greedy tokens and the same logits, and
the expert-sharded MoE (SUM all-reduce of fp32 expert-slice partials) matches the
whole layer.  Skipped on a box with fewer than 2 GPUs.

The ranks are child processes (spawn); each waits only on NCCL collectives with a short
process-group timeout, and the parent joins them with a time limit."""

import os
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rank_main(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta

        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        import flash_next_rtxpro6000_b200 as fx
        from flash_next_rtxpro6000_b200 import sharded
        from flash_next_rtxpro6000_b200 import synthetic as syn
        from flash_next_rtxpro6000_b200.w4a16_nvfp4_gemv import swizzle_blockscale

        fx.prealloc(dev)
        # vocab-sharded head
        V, K, M = 16384, 2048, 4
        head = syn.w8_head(V, K, seed=3)
        x = syn.activations(M, seed=4).to(dev)
        r0, n = sharded.shard_rows(V, world, rank)
        w_sh = head.w[r0:r0 + n].contiguous().to(dev)
        s_sh = head.scale[r0:r0 + n].contiguous().to(dev)
        y, am = sharded.sharded_lm_head_argmax(x, w_sh, s_sh, r0)
        full = sharded.all_gather_logits(y)
        # the same greedy tokens with the exchange inside the GEMV (NVLink peer memory),
        # three calls in a row (epochs 1..3, both key slots)
        ex = sharded.PeerExchange(dev)
        am_p2p = []
        for rep in range(3):
            xr = syn.activations(M, seed=4 + rep).to(dev)
            _, a2 = sharded.vocab_sharded_lm_head(xr, w_sh, s_sh, r0, ex)
            am_p2p.append(a2.cpu())
        from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace
        p2p_err = int(_workspace(dev).error_flag.item())
        ex.close()
        # expert-sharded MoE
        E = 64
        L = syn.moe_layer(E, 2048, 512, seed=5)
        ids, wts = syn.routing(M, E=E, seed=6)
        per = E // world
        sl = slice(rank * per, (rank + 1) * per)
        ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev)
        shared = None
        if rank == 0:
            shared = fx.SharedExpert(L.sh_w13.to(dev), swizzle_blockscale(L.sh_s13.to(dev)),
                                     L.sh_g13.to(dev), L.sh_w2.to(dev),
                                     swizzle_blockscale(L.sh_s2.to(dev)), L.sh_g2.to(dev))
        moe = sharded.expert_sharded_moe(
            hidden_states=x, topk_ids=ids.to(dev), topk_weights=wts.to(dev),
            w13_weight=L.w13[sl].contiguous().to(dev),
            w13_blockscale_swizzled=swizzle_blockscale(L.s13[sl].contiguous().to(dev)),
            w13_weight_scale_2=L.g13[sl].contiguous().to(dev),
            w2_weight=L.w2[sl].contiguous().to(dev),
            w2_blockscale_swizzled=swizzle_blockscale(L.s2[sl].contiguous().to(dev)),
            w2_weight_scale_2=L.g2[sl].contiguous().to(dev), expert_offset=rank * per,
            workspace=ws, shared_expert=shared)
        torch.cuda.synchronize()
        if rank == 0:
            q.put(("ok", am.cpu(), full.cpu(), moe.cpu(), am_p2p, p2p_err))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # report to the parent instead of hanging it
        q.put(("error", traceback.format_exc(), None, None, None, None))


def _single_gpu_reference():
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn
    from flash_next_rtxpro6000_b200.w4a16_nvfp4_gemv import swizzle_blockscale

    dev = torch.device("cuda", 0)
    V, K, M = 16384, 2048, 4
    head = syn.w8_head(V, K, seed=3)
    x = syn.activations(M, seed=4).to(dev)
    am = torch.empty(M, dtype=torch.int64, device=dev)
    y = fx.w8a16_gemv(x, head.w.to(dev), head.scale.to(dev), argmax_out=am)
    am_reps = []
    for rep in range(3):
        a = torch.empty(M, dtype=torch.int64, device=dev)
        fx.w8a16_gemv(syn.activations(M, seed=4 + rep).to(dev), head.w.to(dev),
                      head.scale.to(dev), argmax_out=a)
        am_reps.append(a.cpu())
    E = 64
    L = syn.moe_layer(E, 2048, 512, seed=5)
    ids, wts = syn.routing(M, E=E, seed=6)
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev)
    shared = fx.SharedExpert(L.sh_w13.to(dev), swizzle_blockscale(L.sh_s13.to(dev)),
                             L.sh_g13.to(dev), L.sh_w2.to(dev),
                             swizzle_blockscale(L.sh_s2.to(dev)), L.sh_g2.to(dev))
    moe = fx.draft_moe_gemv(
        hidden_states=x, topk_ids=ids.to(dev), topk_weights=wts.to(dev),
        w13_weight=L.w13.to(dev), w13_blockscale_swizzled=swizzle_blockscale(L.s13.to(dev)),
        w13_weight_scale_2=L.g13.to(dev), w2_weight=L.w2.to(dev),
        w2_blockscale_swizzled=swizzle_blockscale(L.s2.to(dev)), w2_weight_scale_2=L.g2.to(dev),
        workspace=ws, shared_expert=shared, out_f32=True)
    torch.cuda.synchronize()
    return am.cpu(), y.cpu(), moe.cpu(), am_reps


@pytest.mark.skipif(torch.cuda.device_count() < 2 if torch.cuda.is_available() else True,
                    reason="needs 2 GPUs")
def test_two_rank_sharded_head_and_moe():
    import torch.multiprocessing as mp

    am1, y1, moe1, am_reps = _single_gpu_reference()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        status, am, full, moe, am_p2p, p2p_err = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert status == "ok", am
    assert torch.equal(am, am1)
    assert p2p_err == 0
    for got, ref in zip(am_p2p, am_reps):
        assert torch.equal(got, ref)
    # a shard may be tiled differently (its own plan), which can move an fp32 sum by an
    # ulp before the bf16 rounding
    assert float((full.float() - y1.float()).abs().max() / y1.float().abs().max()) <= 2e-2
    assert float((full == y1).float().mean()) > 0.99
    rel = (moe.float() - moe1.bfloat16().float()).abs().max() / moe1.abs().max()
    assert float(rel) <= 1e-2

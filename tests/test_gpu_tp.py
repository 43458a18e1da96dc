"""Tensor parallelism on 2 B200s over NCCL: the block op at TP=2 against TP=1 and the fp32
oracle, and the two-layer golden step at TP=2 against the reference's own output.  Skipped on
boxes with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from oracle import dit_ref as R
        from wanb200 import BlockWeights, FastBlock, FastCrossKV, FastWanDiT, WanSpec, device_error
        from wanb200 import random_block_state
        from wanb200.dit import rope_tables
        out = {}
        # ---- one config-0 block (dim 3072, 24 heads, L = 6x12x15) at TP = world
        spec = WanSpec()
        grid = (6, 12, 15)
        L = 1080
        sd = random_block_state(spec, 11)
        g = torch.Generator().manual_seed(12)
        x = torch.randn(2, L, spec.dim, generator=g).to(torch.bfloat16)
        e0 = torch.randn(1, grid[0], 6, spec.dim, generator=g) * 0.1
        ctx = torch.randn(2, 512, spec.dim, generator=g).to(torch.bfloat16)
        cos, sin = rope_tables(grid, 128, dev)
        w = BlockWeights(sd, spec.num_heads, dev, rank, world)
        ck, cv = FastCrossKV(w, dist.group.WORLD)(ctx.to(dev))
        blk_tp = FastBlock(w, grid[0], dist.group.WORLD)
        y_tp = blk_tp(x.to(dev), e0.to(dev), cos, sin, ck, cv)
        # the whole block as one C call, its all-reduces through the callback into torch.distributed
        from wanb200.block import block_forward_c
        y_c = block_forward_c(blk_tp, x.to(dev), e0.to(dev), cos, sin, ck, cv)
        # one chunk (a single blocking all-reduce per projection) against the overlapped chunks
        y_1 = FastBlock(w, grid[0], dist.group.WORLD, tp_chunks=1)(x.to(dev), e0.to(dev), cos, sin, ck, cv)
        torch.cuda.synchronize()
        out["c_entry_vs_op"] = R.rel_rms(y_c.float().cpu(), y_tp.float().cpu())
        out["chunks_vs_one"] = R.rel_rms(y_1.float().cpu(), y_tp.float().cpu())
        if rank == 0:
            w1 = BlockWeights(sd, spec.num_heads, dev)
            ck1, cv1 = FastCrossKV(w1)(ctx.to(dev))
            y1 = FastBlock(w1, grid[0])(x.to(dev), e0.to(dev), cos, sin, ck1, cv1)
            out["tp_vs_tp1"] = R.rel_rms(y_tp.float().cpu(), y1.float().cpu())
            p32 = {k: v.float() for k, v in sd.items()}
            cosr, sinr = R.rope_tables(R.model_freqs(128), grid, 128)
            ckr, cvr = R.cross_kv(p32, ctx.float(), spec.num_heads)
            y_ref = R.block_fwd(p32, x.float(), e0, cosr, sinr, ckr, cvr, grid[0], spec.num_heads)
            out["tp_vs_oracle"] = R.rel_rms(y_tp.float().cpu(), y_ref)
        # ---- the golden two-layer step at TP = world (2 heads -> 1 per rank)
        mg = torch.load(os.path.join(ROOT, "tests", "golden", "model_small.pt"), weights_only=False)
        cfg = mg["cfg"]
        sp = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"],
                     num_layers=cfg["num_layers"], freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"],
                     in_dim=cfg["in_dim"], out_dim=cfg["out_dim"], text_len=cfg["text_len"])
        lat = mg["latent"]
        fast = FastWanDiT((sp, mg["state_dict"]), (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2), mg["guide"],
                          dev, tp_group=dist.group.WORLD)
        fast.set_context(mg["ctx"].to(dev), mg["ctx_null"].to(dev))
        pred = fast(lat.to(dev), mg["t"])
        out["step_vs_reference"] = R.rel_rms(pred.float().cpu(), mg["noise_pred"])
        # ---- the same step CFG-parallel: rank 0 = cond, rank 1 = uncond, pair all-reduce at the head
        from wanb200.parallel import make_layout
        lay = make_layout("cfg")
        fc = FastWanDiT((sp, mg["state_dict"]), (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2), mg["guide"],
                        dev, cfg_group=lay.cfg_group, pair_group=lay.pair_group, tp_group=lay.tp_group)
        fc.set_context(mg["ctx"].to(dev), mg["ctx_null"].to(dev))
        pc = fc(lat.to(dev), mg["t"])
        out["cfgpar_vs_reference"] = R.rel_rms(pc.float().cpu(), mg["noise_pred"])
        out["device_error"] = device_error(reset=True)
        q.put((rank, out))
    except Exception as ex:  # reported to the parent
        import traceback
        q.put((rank, traceback.format_exc() + repr(ex)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason=f"needs {WORLD} GPUs")
def test_tp2_block_and_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(WORLD):
        assert isinstance(res[r], dict), res[r]
        assert res[r]["device_error"] == 0
        assert res[r]["step_vs_reference"] < 5e-2, res[r]
        assert res[r]["cfgpar_vs_reference"] < 5e-2, res[r]
    print("tp2:", res[0])
    for r in range(WORLD):
        assert res[r]["c_entry_vs_op"] < 1e-3, res[r]
        assert res[r]["chunks_vs_one"] < 1e-3, res[r]
    assert res[0]["tp_vs_tp1"] < 1e-2
    assert res[0]["tp_vs_oracle"] < 2e-2

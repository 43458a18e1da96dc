"""Sequence-parallel layouts on B200s.

Token-sharded residual + local all-head cross-attention (`_FastBlockSP`):
* 2 GPUs: `FastBlockSP` at TP=2, batch 1, on a config-0-sized block (7854-token grid cut to
  6x12x15) against the TP=1 device block and the fp32 oracle;
* 4 GPUs: the two-layer golden step in the CFG-parallel 2 x (SP+TP 2) layout against the
  reference's own ref_fp32.main() output.
Q-local sequence parallelism (`WanSelfAttentionSP`: local queries, K/V all-gathered):
* 2 GPUs: `FastBlock` with a KVGather (peer push and NCCL), batch 2, on the 6x12x15 grid and
  on a 3x7x9 grid whose 189 tokens leave the last shard padded, against the single-GPU block
  and the fp32 oracle;
* 4 / 8 GPUs: the golden step in the "sp", "cfgsp" and "cfgsptp" layouts.
Each test is skipped on boxes with fewer GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    import datetime
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    return dev


def _block_worker(rank, world, port, q, comm_kind):
    try:
        dev = _init(rank, world, port)
        from oracle import dit_ref as R
        from wanb200 import BlockWeights, FastBlock, FastCrossKV, WanSpec, device_error, random_block_state
        from wanb200.block import FastBlockSP
        from wanb200.dit import rope_tables
        spec = WanSpec()
        grid = (6, 12, 15)
        L = 1080
        sd = random_block_state(spec, 21)
        g = torch.Generator().manual_seed(22)
        x = torch.randn(1, L, spec.dim, generator=g).to(torch.bfloat16)
        e0 = torch.randn(1, grid[0], 6, spec.dim, generator=g) * 0.1
        ctx = torch.randn(1, 512, spec.dim, generator=g).to(torch.bfloat16)
        cos, sin = rope_tables(grid, 128, dev)
        w = BlockWeights(sd, spec.num_heads, dev, rank, world, local_cross=True)
        ck, cv = FastCrossKV(w)(ctx.to(dev))
        S = -(-L // world)
        xp = torch.cat([x[0], x.new_zeros(S * world - L, spec.dim)]).to(dev)
        comm = None
        if comm_kind == "peer":
            from wanb200.comm import PeerComm
            comm = PeerComm(dist.group.WORLD, S, spec.dim, dev)
        blk = FastBlockSP(w, L, grid[0], dist.group.WORLD, comm=comm)
        xs = xp[rank * S:(rank + 1) * S].contiguous()
        ys = blk(xs, e0.to(dev), cos, sin, ck, cv)
        ys2 = blk(xs, e0.to(dev), cos, sin, ck, cv)  # the buffers and barrier epochs are reused
        full = torch.empty(S * world, spec.dim, dtype=ys.dtype, device=dev)
        dist.all_gather_into_tensor(full, ys)
        out = {"device_error": device_error(reset=True),
               "repeat": float((ys.float() - ys2.float()).abs().max())}
        if rank == 0:
            y = full[:L].float().cpu()
            w1 = BlockWeights(sd, spec.num_heads, dev)
            ck1, cv1 = FastCrossKV(w1)(ctx.to(dev))
            y1 = FastBlock(w1, grid[0])(x.to(dev), e0.to(dev), cos, sin, ck1, cv1)[0].float().cpu()
            out["sp_vs_tp1"] = R.rel_rms(y, y1)
            p32 = {k: v.float() for k, v in sd.items()}
            cosr, sinr = R.rope_tables(R.model_freqs(128), grid, 128)
            ckr, cvr = R.cross_kv(p32, ctx.float(), spec.num_heads)
            y_ref = R.block_fwd(p32, x.float(), e0, cosr, sinr, ckr, cvr, grid[0], spec.num_heads)[0]
            out["sp_vs_oracle"] = R.rel_rms(y, y_ref)
        q.put((rank, out))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _step_worker(rank, world, port, q):
    try:
        dev = _init(rank, world, port)
        from oracle import dit_ref as R
        from wanb200 import FastWanDiT, WanSpec, device_error
        from wanb200.parallel import make_layout
        mg = torch.load(os.path.join(ROOT, "tests", "golden", "model_small.pt"), weights_only=False)
        cfg = mg["cfg"]
        sp = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"],
                     num_layers=cfg["num_layers"], freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"],
                     in_dim=cfg["in_dim"], out_dim=cfg["out_dim"], text_len=cfg["text_len"])
        lat = mg["latent"]
        lay = make_layout("cfg")
        fc = FastWanDiT((sp, mg["state_dict"]), (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2), mg["guide"],
                        dev, cfg_group=lay.cfg_group, pair_group=lay.pair_group, tp_group=lay.tp_group)
        assert fc.sp
        fc.set_context(mg["ctx"].to(dev), mg["ctx_null"].to(dev))
        pred = fc(lat.to(dev), mg["t"])
        q.put((rank, {"step_vs_reference": R.rel_rms(pred.float().cpu(), mg["noise_pred"]),
                      "device_error": device_error(reset=True)}))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _qsp_block_worker(rank, world, port, q, comm_kind):
    try:
        dev = _init(rank, world, port)
        from oracle import dit_ref as R
        from wanb200 import BlockWeights, FastBlock, FastCrossKV, WanSpec, device_error, random_block_state
        from wanb200.comm import KVGather
        from wanb200.dit import rope_tables
        spec = WanSpec()
        sd = random_block_state(spec, 31)
        w = BlockWeights(sd, spec.num_heads, dev)
        out = {}
        for grid in ((6, 12, 15), (3, 7, 9)):
            L = grid[0] * grid[1] * grid[2]
            g = torch.Generator().manual_seed(L)
            x = torch.randn(2, L, spec.dim, generator=g).to(torch.bfloat16)
            e0 = torch.randn(1, grid[0], 6, spec.dim, generator=g) * 0.1
            ctx = torch.randn(2, 512, spec.dim, generator=g).to(torch.bfloat16)
            cos, sin = rope_tables(grid, 128, dev)
            ck, cv = FastCrossKV(w)(ctx.to(dev))
            kv = KVGather(dist.group.WORLD, 2, L, 2 * spec.dim, dev, comm=comm_kind)
            S = kv.S
            pad = world * S - L
            cosp = torch.cat([cos, cos.new_zeros(1, pad, 1, 64)], dim=1)
            sinp = torch.cat([sin, sin.new_zeros(1, pad, 1, 64)], dim=1)
            xp = torch.cat([x, x.new_zeros(2, pad, spec.dim)], dim=1).to(dev)
            xs = xp[:, rank * S:(rank + 1) * S].contiguous()
            blk = FastBlock(w, grid[0], sp=kv)
            ys = blk(xs, e0.to(dev), cosp, sinp, ck, cv)
            ys2 = blk(xs, e0.to(dev), cosp, sinp, ck, cv)  # second gather buffer, next barrier epoch
            full = torch.empty(world, 2, S, spec.dim, dtype=ys.dtype, device=dev)
            dist.all_gather_into_tensor(full, ys.contiguous())
            tag = f"L{L}"
            out[f"{tag}_repeat"] = float((ys.float() - ys2.float()).abs().max())
            if rank == 0:
                y = full.permute(1, 0, 2, 3).reshape(2, world * S, spec.dim)[:, :L].float().cpu()
                y1 = FastBlock(w, grid[0])(x.to(dev), e0.to(dev), cos, sin, ck, cv).float().cpu()
                out[f"{tag}_vs_single"] = R.rel_rms(y, y1)
                p32 = {k: v.float() for k, v in sd.items()}
                cosr, sinr = R.rope_tables(R.model_freqs(128), grid, 128)
                ckr, cvr = R.cross_kv(p32, ctx.float(), spec.num_heads)
                y_ref = R.block_fwd(p32, x.float(), e0, cosr, sinr, ckr, cvr, grid[0], spec.num_heads)
                out[f"{tag}_vs_oracle"] = R.rel_rms(y, y_ref)
        out["device_error"] = device_error(reset=True)
        q.put((rank, out))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _layout_step_worker(rank, world, port, q, kind, comm_kind):
    try:
        dev = _init(rank, world, port)
        from oracle import dit_ref as R
        from wanb200 import FastWanDiT, WanSpec, device_error
        from wanb200.parallel import make_layout
        mg = torch.load(os.path.join(ROOT, "tests", "golden", "model_small.pt"), weights_only=False)
        cfg = mg["cfg"]
        sp = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"],
                     num_layers=cfg["num_layers"], freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"],
                     in_dim=cfg["in_dim"], out_dim=cfg["out_dim"], text_len=cfg["text_len"])
        lat = mg["latent"]
        lay = make_layout(kind)
        fc = FastWanDiT((sp, mg["state_dict"]), (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2), mg["guide"],
                        dev, cfg_group=lay.cfg_group, pair_group=lay.pair_group, tp_group=lay.tp_group,
                        sp_group=lay.sp_group, comm=comm_kind)
        assert fc.kv_gather is not None and not fc.sp
        fc.set_context(mg["ctx"].to(dev), mg["ctx_null"].to(dev))
        pred = fc(lat.to(dev), mg["t"])
        pred2 = fc(lat.to(dev), mg["t"])
        q.put((rank, {"step_vs_reference": R.rel_rms(pred.float().cpu(), mg["noise_pred"]),
                      "repeat": R.rel_rms(pred2.float().cpu(), pred.float().cpu()),
                      "layout": lay.describe(world), "device_error": device_error(reset=True)}))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(target, world, *extra):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + extra) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert isinstance(res[r], dict), res[r]
        assert res[r]["device_error"] == 0
    return res


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("comm_kind", ["nccl", "peer"])
def test_sp_block_tp2(comm_kind):
    """comm_kind "peer": the all-gathers / reduce-scatters run inside the LayerNorm (row push) and
    the row-parallel GEMM epilogue (inbox scatter) over NVLink peer memory, with peer barriers."""
    res = _run(_block_worker, 2, comm_kind)
    print(f"sp2[{comm_kind}]:", res[0])
    assert res[0]["sp_vs_tp1"] < 1e-2
    assert res[0]["sp_vs_oracle"] < 2e-2
    for r in range(2):
        assert res[r]["repeat"] < 0.1, res[r]  # only the fp32 atomics of the norm sums may differ


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_cfg_parallel_sp_step_4gpu():
    res = _run(_step_worker, 4)
    print("cfg2xsp2:", res)
    for r in range(4):
        assert res[r]["step_vs_reference"] < 5e-2, res[r]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("comm_kind", ["nccl", "peer"])
def test_qlocal_sp_block_2gpu(comm_kind):
    """Q-local SP=2, batch 2: local queries attend the K/V gathered from both ranks (pushed over
    NVLink by wanb200_shard_gather, or NCCL all-gather)."""
    res = _run(_qsp_block_worker, 2, comm_kind)
    print(f"qsp2[{comm_kind}]:", res[0])
    for tag in ("L1080", "L189"):
        assert res[0][f"{tag}_vs_single"] < 1e-2, res[0]
        assert res[0][f"{tag}_vs_oracle"] < 2e-2, res[0]
        for r in range(2):
            assert res[r][f"{tag}_repeat"] < 0.1, res[r]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("kind,comm_kind", [("sp", "peer"), ("cfgsp", "peer"), ("cfgsp", "nccl")])
def test_qlocal_sp_step_4gpu(kind, comm_kind):
    res = _run(_layout_step_worker, 4, kind, comm_kind)
    print(f"{kind}[{comm_kind}]:", res)
    for r in range(4):
        assert res[r]["step_vs_reference"] < 5e-2, res[r]
        assert res[r]["repeat"] < 1e-2, res[r]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_cfg_sp2_tp2_step_8gpu():
    """The config-3 layout: CFG groups of 4 GPUs, each SP2 x TP2."""
    res = _run(_layout_step_worker, 8, "cfgsptp", "peer")
    print("cfgsptp:", res[0])
    for r in range(8):
        assert res[r]["layout"] == "cfg2xsp2xtp2"
        assert res[r]["step_vs_reference"] < 5e-2, res[r]

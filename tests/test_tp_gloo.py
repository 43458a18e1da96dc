"""Tensor-parallel decomposition on CPU ranks (gloo, world size 2 and 4).

Each rank slices the block with the product's `BlockWeights` (the reference's
`shard_model_tp` pattern, models/tp_utils.py:378-458), runs its share with the CPU
restatement `oracle.tp_ref.block_fwd_tp` (same all-reduce points as `FastBlock`'s TP branch)
and must reproduce the unsharded oracle block.  A second test checks that a collective whose
peer has gone away fails with an error inside the process-group timeout instead of hanging.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port, timeout_s=60):
    import datetime
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _tp_worker(rank, world, port, q):
    try:
        _setup(rank, world, port)
        torch.set_num_threads(1)
        from oracle import dit_ref as R
        from oracle.tp_ref import block_fwd_tp
        from wanb200 import BlockWeights, WanSpec, random_block_state
        spec = WanSpec(dim=512, ffn_dim=1024, num_heads=4)
        grid = (2, 3, 4)
        B, L, Lc = 2, 24, 16
        sd = random_block_state(spec, 5)
        g = torch.Generator().manual_seed(9)
        x = torch.randn(B, L, spec.dim, generator=g)
        e0 = torch.randn(1, grid[0], 6, spec.dim, generator=g) * 0.1
        ctx = torch.randn(B, Lc, spec.dim, generator=g)
        cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
        p32 = {k: v.float() for k, v in sd.items()}
        ck, cv = R.cross_kv(p32, ctx, spec.num_heads)  # all heads
        w = BlockWeights(sd, spec.num_heads, "cpu", rank, world)
        hs = slice(rank * w.local_heads, (rank + 1) * w.local_heads)
        y = block_fwd_tp(w, x, e0, cos, sin, ck[:, :, hs].contiguous(), cv[:, :, hs].contiguous(), grid[0],
                         lambda t: dist.all_reduce(t))
        y_ref = R.block_fwd(p32, x, e0, cos, sin, ck, cv, grid[0], spec.num_heads)
        q.put((rank, R.rel_rms(y, y_ref)))
    except Exception as ex:  # pragma: no cover - reported to the parent
        q.put((rank, repr(ex)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_decomposition_matches_unsharded_oracle(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-5, (r, res[r])


def _lost_peer_worker(rank, world, port, q):
    try:
        _setup(rank, world, port, timeout_s=5)
        t = torch.ones(4)
        dist.all_reduce(t)  # both ranks take part
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before leaving
            os._exit(0)  # leaves between steps, nothing in flight
        try:
            dist.all_reduce(t)  # the peer is gone: must raise, not hang
            q.put((rank, "no error"))
        except Exception as ex:
            q.put((rank, "raised:" + type(ex).__name__))
    except Exception as ex:  # pragma: no cover
        q.put((rank, repr(ex)))


def test_collective_with_lost_peer_raises_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lost_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("raised:"), res[0]


def _layout_worker(rank, world, port, q):
    try:
        _setup(rank, world, port)
        from wanb200.parallel import make_layout
        lay = make_layout("cfg")
        t = torch.tensor([float(rank)])
        dist.all_reduce(t, group=lay.tp_group)
        p = torch.tensor([float(rank)])
        dist.all_reduce(p, group=lay.pair_group)
        q.put((rank, (lay.cfg_group, lay.tp_size, float(t), float(p), lay.describe(world))))
    except Exception as ex:  # pragma: no cover
        q.put((rank, repr(ex)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_cfg_parallel_layout_groups():
    """4 ranks: CFG groups {0,1} (cond) and {2,3} (uncond) with TP 2 inside, pairs {0,2}, {1,3}
    (the reference's CFG-parallel split, inference_neuron_ti2v.py:241-274)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_layout_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res[0] == (0, 2, 1.0, 2.0, "cfg2x(sp+tp)2"), res[0]
    assert res[1] == (0, 2, 1.0, 4.0, "cfg2x(sp+tp)2"), res[1]
    assert res[2] == (1, 2, 5.0, 2.0, "cfg2x(sp+tp)2"), res[2]
    assert res[3] == (1, 2, 5.0, 4.0, "cfg2x(sp+tp)2"), res[3]


def _sp_worker(rank, world, port, q):
    try:
        _setup(rank, world, port)
        torch.set_num_threads(1)
        from oracle import dit_ref as R
        from oracle.tp_ref import block_fwd_sp
        from wanb200 import BlockWeights, WanSpec, random_block_state
        spec = WanSpec(dim=512, ffn_dim=1024, num_heads=4)
        grid = (2, 3, 5)
        L, Lc = 30, 16  # 30 tokens over `world` ranks: padded when world does not divide 30
        sd = random_block_state(spec, 6)
        g = torch.Generator().manual_seed(10)
        x = torch.randn(1, L, spec.dim, generator=g)
        e0 = torch.randn(1, grid[0], 6, spec.dim, generator=g) * 0.1
        ctx = torch.randn(1, Lc, spec.dim, generator=g)
        cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
        p32 = {k: v.float() for k, v in sd.items()}
        ck, cv = R.cross_kv(p32, ctx, spec.num_heads)
        y_ref = R.block_fwd(p32, x, e0, cos, sin, ck, cv, grid[0], spec.num_heads)[0]
        S = -(-L // world)
        xp = torch.cat([x[0], x.new_zeros(S * world - L, spec.dim)])
        xs = xp[rank * S:(rank + 1) * S].contiguous()
        w = BlockWeights(sd, spec.num_heads, "cpu", rank, world, local_cross=True)

        def ag(t):
            out = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(out, t.contiguous())
            return torch.cat(out)

        def rs(t):
            t = t.contiguous()
            dist.all_reduce(t)
            return t[rank * S:(rank + 1) * S]

        ys = block_fwd_sp(w, xs, e0, cos, sin, ck, cv, L, grid[0], rank, world, ag, rs, lambda t: dist.all_reduce(t))
        y = ag(ys)[:L]
        q.put((rank, R.rel_rms(y, y_ref)))
    except Exception as ex:  # pragma: no cover
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_parallel_decomposition_matches_unsharded_oracle(world):
    """Token-sharded residual + all-gather / reduce-scatter around the TP GEMMs + local
    all-head cross-attention (the reference's _FastBlockSP with full_cross) == one block."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-5, (r, res[r])


def _qsp_worker(rank, world, port, q, tp):
    try:
        _setup(rank, world, port)
        torch.set_num_threads(1)
        from oracle import dit_ref as R
        from oracle.tp_ref import block_fwd_qsp
        from wanb200 import BlockWeights, WanSpec, random_block_state
        sp = world // tp
        # contiguous TP groups, SP groups strided across them (parallel_state.py's tp / attn-sp)
        tp_groups = [dist.new_group(list(range(j * tp, (j + 1) * tp))) for j in range(sp)]
        sp_groups = [dist.new_group([i + j * tp for j in range(sp)]) for i in range(tp)]
        tp_group, sp_group = tp_groups[rank // tp], sp_groups[rank % tp]
        sp_rank, tp_rank = rank // tp, rank % tp
        spec = WanSpec(dim=512, ffn_dim=1024, num_heads=4)
        grid = (2, 3, 5)
        L, Lc, B = 30, 16, 2  # 30 tokens over 4 SP ranks: shards of 8, the last one padded by 2
        sd = random_block_state(spec, 7)
        g = torch.Generator().manual_seed(11)
        x = torch.randn(B, L, spec.dim, generator=g)
        e0 = torch.randn(1, grid[0], 6, spec.dim, generator=g) * 0.1
        ctx = torch.randn(B, Lc, spec.dim, generator=g)
        cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
        p32 = {k: v.float() for k, v in sd.items()}
        ck, cv = R.cross_kv(p32, ctx, spec.num_heads)
        y_ref = R.block_fwd(p32, x, e0, cos, sin, ck, cv, grid[0], spec.num_heads)
        S = -(-L // sp)
        pad = S * sp - L
        xs = torch.cat([x, x.new_zeros(B, pad, spec.dim)], dim=1)[:, sp_rank * S:(sp_rank + 1) * S].contiguous()
        cosp = torch.cat([cos, cos.new_zeros(1, pad, 1, 64)], dim=1)
        sinp = torch.cat([sin, sin.new_zeros(1, pad, 1, 64)], dim=1)
        w = BlockWeights(sd, spec.num_heads, "cpu", tp_rank, tp)
        nl = w.local_heads
        ckl = ck[:, :, tp_rank * nl:(tp_rank + 1) * nl].contiguous()
        cvl = cv[:, :, tp_rank * nl:(tp_rank + 1) * nl].contiguous()

        def gather(t):
            out = [torch.empty_like(t) for _ in range(sp)]
            dist.all_gather(out, t.contiguous(), group=sp_group)
            return torch.cat(out, dim=1)

        def ar(t):
            if tp > 1:
                dist.all_reduce(t, group=tp_group)

        ys = block_fwd_qsp(w, xs, e0, cosp, sinp, ckl, cvl, L, grid[0], sp_rank, sp, gather, ar)
        y = gather(ys)[:, :L]
        q.put((rank, R.rel_rms(y, y_ref)))
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world,tp", [(2, 1), (4, 1), (4, 2)])
def test_qlocal_sequence_parallel_decomposition_matches_unsharded_oracle(world, tp):
    """Whole block on each rank's token shard (batch 2), K/V all-gathered over the SP group for
    the local queries, TP inside (the reference's WanSelfAttentionSP layout) == one block."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_qsp_worker, args=(r, world, port, q, tp)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-5, (r, res[r])


def _qsp_layout_worker(rank, world, port, q, kind):
    try:
        _setup(rank, world, port)
        from wanb200.parallel import make_layout
        lay = make_layout(kind)
        t = torch.tensor([float(rank)])
        dist.all_reduce(t, group=lay.sp_group)
        p = torch.tensor([float(rank)])
        if lay.pair_group is not None:
            dist.all_reduce(p, group=lay.pair_group)
        q.put((rank, (lay.cfg_group, lay.sp_size, lay.tp_size, float(t), float(p), lay.describe(world))))
    except Exception as ex:  # pragma: no cover
        q.put((rank, repr(ex)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["sp", "cfgsp", "cfgsptp"])
def test_qlocal_layout_groups(kind):
    """4 ranks: "sp" = one SP group of all ranks; "cfgsp" / "cfgsptp" (TP 1 at 4 ranks) = CFG
    groups {0,1} and {2,3} each one SP group, pairs {0,2}, {1,3}."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_qsp_layout_worker, args=(r, 4, port, q, kind)) for r in range(4)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    if kind == "sp":
        for r in range(4):
            assert res[r] == (None, 4, 1, 6.0, float(r), "sp4"), res[r]
        return
    name = "cfg2xsp2" if kind == "cfgsp" else "cfg2xsp2xtp1"
    assert res[0] == (0, 2, 1, 1.0, 2.0, name), res[0]
    assert res[1] == (0, 2, 1, 1.0, 4.0, name), res[1]
    assert res[2] == (1, 2, 1, 5.0, 2.0, name), res[2]
    assert res[3] == (1, 2, 1, 5.0, 4.0, name), res[3]

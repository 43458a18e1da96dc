"""Generate the golden fixtures that pin `oracle/dit_ref.py` to the reference itself.

Run in a container that has the reference checkout (yahavb/wan2-ti2v-5b) at REF_ROOT:

    python tests/golden/make_golden.py [REF_ROOT]

It imports the reference's own modules (with two import shims: a `diffusers` stub, since
`WanModel` only needs `ConfigMixin`/`register_to_config`/`ModelMixin`, and bare namespace
packages for `wan` / `wan.modules` so `wan/__init__.py`, which needs `easydict`, is skipped),
builds a small seeded WanModel (dim 256 = 2 heads x 128, ffn 512, 2 layers, text_dim 64),
and records:

  * model_small.pt -- the bf16-exact weights, the step-0 inputs and the reference's own
    `scripts/validate/ref_fp32.py:main()` output (noise_pred), run unmodified on a
    synthetic `step0.pt` dump with `WanModel.from_pretrained` pointed at the small model;
  * block_small.pt -- block 0 of that model (weights: model_small.pt) through `ref_fp32.block_fwd` (x, e0, cos, sin, ck, cv -> y),
    plus the reference's bf16 `WanAttentionBlock.forward` and bf16 `_FastBlock.forward`
    outputs on the same inputs (calibration of the reference's own bf16 error);
  * rope_small.pt -- `fast_dit._rope_tables` for small grids and strided rows of the three
    benchmark grids (6x12x15, 21x17x22, 31x22x40), and `fast_dit._rope` on a random tensor;
  * unipc_small.pt -- the reference's sampler, `FlowUniPCMultistepScheduler`
    (wan/utils/fm_solvers_unipc.py) constructed and stepped as inference_neuron_ti2v.py:497-532
    does, on seeded latents and model outputs (fp32 and bf16; shift 5 and 1; 10 and 3 steps).
    `--unipc-only` regenerates just this file.

The GPU box never runs this script (the reference is not there); the fixtures travel.
"""
import importlib.util
import os
import sys
import tempfile
import types

import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
_ARGS = [a for a in sys.argv[1:] if not a.startswith("--")]
REF = _ARGS[0] if _ARGS else os.environ.get("WAN_REF_ROOT", "")
if not REF:
    raise SystemExit("usage: python tests/golden/make_golden.py REF_ROOT [--unipc-only]  "
                     "(or set WAN_REF_ROOT): the path of the reference checkout")

DIM, FFN, HEADS, LAYERS, TEXT_DIM, FREQ_DIM, IN_DIM, LC = 256, 512, 2, 2, 64, 256, 48, 16
GRID_LATENT = (2, 6, 8)  # latent [48, F, H, W] -> token grid (2, 3, 4), L = 24
T_STEP = 500.0


def import_reference():
    sys.path.insert(0, REF)
    d = types.ModuleType("diffusers")
    cu = types.ModuleType("diffusers.configuration_utils")

    class ConfigMixin:  # WanModel only subclasses it
        pass

    cu.ConfigMixin = ConfigMixin
    cu.register_to_config = lambda f: f
    dm = types.ModuleType("diffusers.models")
    mu = types.ModuleType("diffusers.models.modeling_utils")
    mu.ModelMixin = nn.Module
    sys.modules.update({"diffusers": d, "diffusers.configuration_utils": cu,
                        "diffusers.models": dm, "diffusers.models.modeling_utils": mu})
    for name, path in (("wan", os.path.join(REF, "wan")), ("wan.modules", os.path.join(REF, "wan/modules"))):
        m = types.ModuleType(name)
        m.__path__ = [path]
        sys.modules[name] = m
    import wan.modules.model as M
    import models.fast_dit as fd
    spec = importlib.util.spec_from_file_location("ref_fp32", os.path.join(REF, "scripts/validate/ref_fp32.py"))
    rf = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rf)
    return M, fd, rf


def seeded_model(M):
    torch.manual_seed(0)
    model = M.WanModel(model_type="ti2v", patch_size=(1, 2, 2), text_len=LC, in_dim=IN_DIM, dim=DIM,
                       ffn_dim=FFN, freq_dim=FREQ_DIM, text_dim=TEXT_DIM, out_dim=IN_DIM,
                       num_heads=HEADS, num_layers=LAYERS, cross_attn_norm=True, eps=1e-6)
    g = torch.Generator().manual_seed(1234)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name and name.endswith("weight"):
                v = 1.0 + 0.1 * torch.randn(p.shape, generator=g)
            elif name.endswith("modulation"):
                v = torch.randn(p.shape, generator=g) / DIM ** 0.5
            elif name.endswith("bias"):
                v = 0.02 * torch.randn(p.shape, generator=g)
            else:
                v = 0.02 * torch.randn(p.shape, generator=g)
            p.copy_(v.to(torch.bfloat16).float())  # bf16-exact, so the device weights equal these
    return model.eval().float()


def main():
    torch.set_grad_enabled(False)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    M, fd, rf = import_reference()
    model = seeded_model(M)
    sd = {k: v.to(torch.bfloat16) for k, v in model.state_dict().items()}
    cfg = dict(num_heads=HEADS, num_layers=LAYERS, freq_dim=FREQ_DIM, patch=(1, 2, 2), out_dim=IN_DIM,
               dim=DIM, ffn_dim=FFN, text_dim=TEXT_DIM, in_dim=IN_DIM, text_len=LC)

    g = torch.Generator().manual_seed(7)
    latent = torch.randn((IN_DIM,) + GRID_LATENT, generator=g).to(torch.bfloat16).float()
    ctx = torch.randn(LC, TEXT_DIM, generator=g).to(torch.bfloat16).float()
    ctx_null = torch.randn(LC, TEXT_DIM, generator=g).to(torch.bfloat16).float()

    # ---- the reference's own ref_fp32.main() on a synthetic step0 dump
    M.WanModel.from_pretrained = classmethod(lambda cls, path: model)
    with tempfile.TemporaryDirectory() as tmp:
        src, out = os.path.join(tmp, "dump"), os.path.join(tmp, "out")
        os.makedirs(src)
        torch.save({"latent_in": latent, "t": T_STEP, "ctx": ctx, "ctx_null": ctx_null,
                    "noise_pred": torch.zeros(IN_DIM, *GRID_LATENT)}, os.path.join(src, "step0.pt"))
        argv = sys.argv
        sys.argv = ["ref_fp32.py", src, out]
        os.environ.setdefault("THREADS", str(max(1, os.cpu_count() or 1)))
        rf.main()
        sys.argv = argv
        noise_pred = torch.load(os.path.join(out, "ref_fp32.pt"))["noise_pred"]
    torch.save({"cfg": cfg, "state_dict": sd, "latent": latent, "t": T_STEP, "ctx": ctx,
                "ctx_null": ctx_null, "guide": rf.GUIDE, "noise_pred": noise_pred.float()},
               os.path.join(HERE, "model_small.pt"))

    # ---- one block: ref_fp32.block_fwd on block 0 with inputs built as ref_fp32.main builds them
    nf, H, W = GRID_LATENT[0], GRID_LATENT[1] // 2, GRID_LATENT[2] // 2
    grid = (nf, H, W)
    L = nf * H * W
    d = DIM // HEADS
    cos, sin = fd._rope_tables(model.freqs, grid, d, torch.device("cpu"))
    t_frames = torch.full((nf,), T_STEP, dtype=torch.float64)
    t_frames[0] = 0.0
    e = model.time_embedding(M.sinusoidal_embedding_1d(model.freq_dim, t_frames).float().unsqueeze(0))
    e0 = model.time_projection(e).unflatten(2, (6, model.dim))
    context = model.text_embedding(torch.stack([ctx, ctx_null], 0).float())
    blk = model.blocks[0]
    ca = blk.cross_attn
    ck = rf.rms(rf.lin(context, ca.k), ca.norm_k).view(2, -1, ca.num_heads, ca.head_dim)
    cv = rf.lin(context, ca.v).view(2, -1, ca.num_heads, ca.head_dim)
    x = torch.randn(2, L, DIM, generator=g).to(torch.bfloat16).float()
    y = rf.block_fwd(blk, x, e0, cos, sin, ck, cv, nf)

    # calibration: the reference's bf16 block paths on the same inputs
    import copy
    from models.tp_utils import shard_model_tp
    blk16 = copy.deepcopy(blk).to(torch.bfloat16)
    e_tok = e0.to(torch.bfloat16).repeat_interleave(H * W, dim=1)  # [1, L, 6, C] per-token
    y_wan16 = blk16(x.to(torch.bfloat16), e_tok, torch.tensor([L, L]), torch.tensor([list(grid)] * 2),
                    model.freqs, context.to(torch.bfloat16), None).float()
    m16 = copy.deepcopy(model)
    shard_model_tp(m16, 0, 1)
    fb = fd._FastBlock(m16.blocks[0].to(torch.bfloat16), nf, "sdpa", None)
    y_fast16 = fb(x.to(torch.bfloat16), e0.to(torch.bfloat16), cos, sin, ck.to(torch.bfloat16),
                  cv.to(torch.bfloat16)).float()
    torch.save({"num_heads": HEADS, "grid": grid, "block_prefix": "blocks.0.", "x": x, "e0": e0.float(), "e": e.float(),
                "cos": cos, "sin": sin, "context": context.float(), "ck": ck.float(), "cv": cv.float(),
                "y": y.float(), "y_wan_bf16": y_wan16, "y_fast_bf16": y_fast16},
               os.path.join(HERE, "block_small.pt"))

    # ---- RoPE tables and rotation
    tables = {}
    for gr in [(2, 3, 4), (3, 5, 7)]:
        c_, s_ = fd._rope_tables(model.freqs, gr, d, torch.device("cpu"))
        tables[gr] = (c_, s_, None)
    full_freqs = M.WanModel.__new__(M.WanModel)  # freqs only depend on head_dim 128
    freqs128 = torch.cat([M.rope_params_neuron(1024, d - 4 * (d // 6)), M.rope_params_neuron(1024, 2 * (d // 6)),
                          M.rope_params_neuron(1024, 2 * (d // 6))], dim=1)
    del full_freqs
    for gr in [(6, 12, 15), (21, 17, 22), (31, 22, 40)]:
        c_, s_ = fd._rope_tables(freqs128, gr, d, torch.device("cpu"))
        rows = torch.arange(0, c_.shape[1], 37)
        tables[gr] = (c_[:, rows], s_[:, rows], rows)
    xr = torch.randn(2, 24, 2, d, generator=g)
    c24, s24 = fd._rope_tables(model.freqs, (2, 3, 4), d, torch.device("cpu"))
    torch.save({"freqs": model.freqs.float(), "tables": tables, "x": xr, "rope_x": fd._rope(xr, c24, s24)},
               os.path.join(HERE, "rope_small.pt"))
    for f in ("model_small.pt", "block_small.pt", "rope_small.pt"):
        print(f, os.path.getsize(os.path.join(HERE, f)))


def import_reference_scheduler():
    """FlowUniPCMultistepScheduler with a `diffusers` stub for its base classes: the config
    decorator records the constructor arguments as `self.config`, as diffusers' does."""
    import functools
    import inspect
    cu = types.ModuleType("diffusers.configuration_utils")

    class ConfigMixin:
        def register_to_config(self, **kw):
            for k, v in kw.items():
                setattr(self.config, k, v)

    def register_to_config(init):
        sig = inspect.signature(init)

        @functools.wraps(init)
        def wrapper(self, *args, **kwargs):
            bound = sig.bind(self, *args, **kwargs)
            bound.apply_defaults()
            cfg = dict(bound.arguments)
            cfg.pop("self")
            self.config = types.SimpleNamespace(**cfg)
            init(self, *args, **kwargs)
        return wrapper

    cu.ConfigMixin, cu.register_to_config = ConfigMixin, register_to_config
    su = types.ModuleType("diffusers.schedulers.scheduling_utils")
    su.KarrasDiffusionSchedulers = []
    su.SchedulerMixin = type("SchedulerMixin", (), {})
    su.SchedulerOutput = lambda prev_sample: types.SimpleNamespace(prev_sample=prev_sample)
    du = types.ModuleType("diffusers.utils")
    du.deprecate = lambda *a, **k: None
    du.is_scipy_available = lambda: False
    saved = {k: sys.modules.get(k) for k in ("diffusers", "diffusers.configuration_utils", "diffusers.schedulers",
                                              "diffusers.schedulers.scheduling_utils", "diffusers.utils")}
    sys.modules.update({"diffusers": types.ModuleType("diffusers"), "diffusers.configuration_utils": cu,
                        "diffusers.schedulers": types.ModuleType("diffusers.schedulers"),
                        "diffusers.schedulers.scheduling_utils": su, "diffusers.utils": du})
    try:
        spec = importlib.util.spec_from_file_location("ref_fm_solvers_unipc",
                                                      os.path.join(REF, "wan/utils/fm_solvers_unipc.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return mod.FlowUniPCMultistepScheduler


def unipc_golden():
    Sched = import_reference_scheduler()
    cases = []
    small, tiny = (1, 48, 2, 4, 6), (1, 48, 1, 2, 2)
    for dtype, shift, steps, shape in ((torch.float32, 5.0, 10, small), (torch.float32, 1.0, 10, small),
                                       (torch.bfloat16, 5.0, 10, small), (torch.float32, 5.0, 3, small),
                                       # the pipeline's default 50 steps, a 2-step (first-order only)
                                       # schedule, and a bf16 latent over 25 steps at shift 3
                                       (torch.float32, 5.0, 50, tiny), (torch.float32, 5.0, 2, tiny),
                                       (torch.bfloat16, 3.0, 25, tiny)):
        s = Sched(num_train_timesteps=1000, shift=1, use_dynamic_shifting=False)
        s.set_timesteps(steps, device=torch.device("cpu"), shift=shift)
        g = torch.Generator().manual_seed(len(cases))
        x = torch.randn(shape, generator=g).to(dtype)
        x_init, outs, mos = x.clone(), [], []
        for i, t in enumerate(s.timesteps):
            mo = (torch.randn(shape, generator=g) * 0.7 + 0.1 * i).to(dtype)
            x = s.step(mo, t, x, return_dict=False)[0]
            mos.append(mo)
            outs.append(x.clone())
        cases.append({"dtype": str(dtype), "shift": shift, "steps": steps, "timesteps": s.timesteps.clone(),
                      "sigmas": s.sigmas.clone(), "x_init": x_init, "model_outputs": mos, "outputs": outs})
    torch.save({"cases": cases}, os.path.join(HERE, "unipc_small.pt"))
    print("unipc_small.pt", os.path.getsize(os.path.join(HERE, "unipc_small.pt")))


if __name__ == "__main__":
    if "--unipc-only" in sys.argv:
        unipc_golden()
    else:
        main()
        unipc_golden()

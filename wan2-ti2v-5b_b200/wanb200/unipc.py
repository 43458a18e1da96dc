"""The denoise loop around the DiT step: multistep UniPC for flow matching, on device tensors.

The reference samples with `FlowUniPCMultistepScheduler` (wan/utils/fm_solvers_unipc.py, the
diffusers 0.31 UniPC converted to flow matching) constructed as
`(num_train_timesteps=1000, shift=1, use_dynamic_shifting=False)` and
`set_timesteps(steps, shift=sample_shift)` (inference_neuron_ti2v.py:497-502), i.e. solver order 2,
B(h) = expm1 ("bh2"), x0 prediction of a flow-matching model output, lower order at the last
step, final sigma 0.  `models/device_unipc.py` keeps its tensor math on the device so the loop
has no host round trip; `FlowUniPC` does the same here:

  * the scalar coefficients (sigmas, log-SNR steps h, expm1 terms, the 2x2 corrector system)
    are computed on the host as 0-dim fp32 tensors, in the reference's arithmetic;
  * the sample and model-output combinations run on the tensors' device, in the reference's
    operation order, with the same scalar x tensor type promotion (a 0-dim fp32 CPU tensor
    times the sample), so on the CPU the result equals the reference bit for bit
    (tests/test_unipc.py against tests/golden/unipc_small.pt).

`denoise()` is the loop of inference_neuron_ti2v.py:505-532 with the scheduler on the device:
noise_pred = DiT(latent, t), latent = step(noise_pred, latent), then the image frame is pinned
back to the image latent (`(1 - mask2) * z_img + mask2 * latent` with mask2 zero on frame 0).
"""
from __future__ import annotations

import numpy as np
import torch

F32 = torch.float32


def _alpha_sigma(sigma):
    return 1 - sigma, sigma


def _log_snr(sigma):
    """lambda = log(alpha) - log(sigma) for a 0-dim fp32 sigma (inf at sigma = 0)."""
    alpha, sigma = _alpha_sigma(sigma)
    return torch.log(alpha) - torch.log(sigma), alpha, sigma


class FlowUniPC:
    """Multistep UniPC (order 2, bh2, x0 prediction, flow-matching outputs) with the state kept
    on the sample's device.  Call `set_timesteps`, then `step` once per timestep in order."""

    def __init__(self, num_train_timesteps: int = 1000, order: int = 2):
        if order != 2:
            raise ValueError("FlowUniPC implements the reference's solver_order 2")
        self.T = num_train_timesteps
        self.order = order
        # training sigmas 1 - linspace(1, 1/T, T) reversed, shift 1 (the constructor's shift)
        alphas = np.linspace(1, 1 / num_train_timesteps, num_train_timesteps)[::-1].copy()
        sig = torch.from_numpy(1.0 - alphas).to(F32)
        self.sigma_max = sig[0].item()
        self.sigma_min = sig[-1].item()
        self.sigmas = None
        self.timesteps = None

    def set_timesteps(self, steps: int, shift: float = 5.0):
        """`steps` sigmas evenly spaced from sigma_max to sigma_min (exclusive), time-shifted by
        shift * s / (1 + (shift - 1) s), plus a final 0; timesteps = int(sigma * T)."""
        s = np.linspace(self.sigma_max, self.sigma_min, steps + 1).copy()[:-1]
        s = shift * s / (1 + (shift - 1) * s)
        self.timesteps = torch.from_numpy(s * self.T).to(torch.int64)
        self.sigmas = torch.from_numpy(np.concatenate([s, [0.0]]).astype(np.float32))
        self.steps = steps
        self.index = 0
        self.x0 = [None, None]  # converted model outputs of the last two steps (oldest first)
        self.lower_order_nums = 0
        self.this_order = 1
        self.last_sample = None

    # ------------------------------------------------------------------ the two updates
    def _coefficients(self, sigma_t, sigma_s0):
        lambda_t, alpha_t, sigma_t = _log_snr(sigma_t)
        lambda_s0, _, sigma_s0 = _log_snr(sigma_s0)
        h = lambda_t - lambda_s0
        hh = -h
        h_phi_1 = torch.expm1(hh)
        return dict(alpha_t=alpha_t, sigma_t=sigma_t, sigma_s0=sigma_s0, lambda_s0=lambda_s0, h=h, hh=hh,
                    h_phi_1=h_phi_1, B_h=torch.expm1(hh))

    def _predict(self, x, order):
        """UniP: the sample at sigmas[index + 1] from the sample at sigmas[index]."""
        i = self.index
        c = self._coefficients(self.sigmas[i + 1], self.sigmas[i])
        m0 = self.x0[-1]
        x_t = c["sigma_t"] / c["sigma_s0"] * x - c["alpha_t"] * c["h_phi_1"] * m0
        if order == 2:
            lambda_s1, _, _ = _log_snr(self.sigmas[i - 1])
            rk = (lambda_s1 - c["lambda_s0"]) / c["h"]
            d1 = (self.x0[-2] - m0) / rk
            rho = float(torch.tensor([0.5], dtype=x.dtype)[0])  # the reference's order-2 simplification
            x_t = x_t - c["alpha_t"] * c["B_h"] * (rho * d1)
        else:
            x_t = x_t - c["alpha_t"] * c["B_h"] * 0
        return x_t.to(x.dtype)

    def _correct(self, x0_now, last_sample, order):
        """UniC: refine the predicted sample at sigmas[index] with the model output there."""
        i = self.index
        c = self._coefficients(self.sigmas[i], self.sigmas[i - 1])
        m0 = self.x0[-1]
        x = last_sample
        hh = c["hh"]
        if order == 1:
            rhos = torch.tensor([0.5], dtype=x.dtype)
            corr = 0
        else:
            lambda_s1, _, _ = _log_snr(self.sigmas[i - 2])
            rk = (lambda_s1 - c["lambda_s0"]) / c["h"]
            d1 = (self.x0[-2] - m0) / rk
            # R rho = b with R rows rk^0, rk^1 over (rk, 1) and b_k = k! phi_{k+1}(hh) hh / B_h
            R = torch.stack([torch.tensor([rk, 1.0]).pow(0), torch.tensor([rk, 1.0]).pow(1)])
            phi = c["h_phi_1"] / hh - 1
            b1 = phi * 1 / c["B_h"]
            phi = phi / hh - 1 / 2
            b2 = phi * 2 / c["B_h"]
            rhos = torch.linalg.solve(R, torch.tensor([b1, b2])).to(x.dtype)
            corr = rhos[0] * d1
        d1_t = x0_now - m0
        x_t = c["sigma_t"] / c["sigma_s0"] * x - c["alpha_t"] * c["h_phi_1"] * m0
        x_t = x_t - c["alpha_t"] * c["B_h"] * (corr + rhos[-1] * d1_t)
        return x_t.to(x.dtype)

    # ------------------------------------------------------------------ one sampler step
    def step(self, model_output: torch.Tensor, sample: torch.Tensor) -> torch.Tensor:
        """model_output: the CFG-combined flow prediction at timesteps[index]; sample: the latent
        there.  Returns the latent at the next timestep."""
        if self.sigmas is None:
            raise RuntimeError("call set_timesteps() first")
        if self.index >= self.steps:
            raise RuntimeError("all timesteps have been stepped")
        i = self.index
        x0 = sample - self.sigmas[i] * model_output
        if i > 0 and self.last_sample is not None:
            sample = self._correct(x0, self.last_sample, self.this_order)
        self.x0 = [self.x0[1], x0]
        order = min(self.order, self.steps - i)  # lower order at the final step
        self.this_order = min(order, self.lower_order_nums + 1)  # and while the history fills
        self.last_sample = sample
        out = self._predict(sample, self.this_order)
        self.lower_order_nums = min(self.lower_order_nums + 1, self.order)
        self.index += 1
        return out


def denoise(dit, latent: torch.Tensor, steps: int, shift: float = 5.0, image_latent: torch.Tensor = None,
            sampler: FlowUniPC = None) -> torch.Tensor:
    """The reference's denoise loop (inference_neuron_ti2v.py:505-532, device scheduler) with
    `dit(latent, t)` the CFG noise prediction (`FastWanDiT.__call__`).  When `dit` has
    `check_device_errors` (FastWanDiT does), the loop ends with it: a bounded wait that expired
    inside a kernel raises WanB200Error instead of returning a silently wrong latent.

    latent [C, F, H, W] on the device; image_latent [C, 1, H, W] (optional): frame 0 is pinned to
    it after every step.  Returns the final latent."""
    s = sampler or FlowUniPC()
    s.set_timesteps(steps, shift)
    if image_latent is not None:
        latent = latent.clone()
        latent[:, :1] = image_latent.to(latent.dtype)
    for t in s.timesteps:
        noise = dit(latent, float(t))
        latent = s.step(noise.reshape(latent.shape).to(latent.dtype), latent)
        if image_latent is not None:
            latent[:, :1] = image_latent.to(latent.dtype)
    check = getattr(dit, "check_device_errors", None)
    if check is not None:  # the loop's result is only valid if no kernel's bounded wait expired
        check()
    return latent

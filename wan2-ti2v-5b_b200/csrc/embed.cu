// The data movement around the DiT's embedding and head GEMMs (models/fast_dit.py:527-545,
// 480-524): the Conv3d patchify of the latent as a gather into the patch-embedding GEMM's rows,
// and the unpatchify of the head's output with the classifier-free-guidance combine.  Both are
// small (6 MB of latent / prediction per step) gathers; the arithmetic around them runs in the
// tcgen05 GEMM (patch / head Linear) and the LayerNorm kernel (head norm + modulation).
#include "common.cuh"
#include "internal.h"

namespace wanb200 {

struct PatchArgs {
  const void* latent;
  int latent_f32;
  int C, F, H, W;     // latent [C, F, H, W]
  int pf, ph, pw;     // patch
  int Fg, Hg, Wg;     // token grid
  int K;              // C * pf * ph * pw
  int batch;
  __nv_bfloat16* out;  // [batch, L, K]
};

// Thread = one element (token l, patch entry k) of the patch matrix, written to every batch copy.
// k follows the Conv3d weight's flattening [C_out, C_in, pf, ph, pw]: k = ((c*pf + i)*ph + j)*pw + u.
__global__ void __launch_bounds__(256) patchify_kernel(const PatchArgs a) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t L = (int64_t)a.Fg * a.Hg * a.Wg;
  if (idx >= L * a.K) return;
  const int l = (int)(idx / a.K), k = (int)(idx - (int64_t)l * a.K);
  const int w = l % a.Wg, h = (l / a.Wg) % a.Hg, f = l / (a.Wg * a.Hg);
  const int u = k % a.pw, j = (k / a.pw) % a.ph, i = (k / (a.pw * a.ph)) % a.pf, c = k / (a.pw * a.ph * a.pf);
  const int64_t src = (((int64_t)c * a.F + f * a.pf + i) * a.H + h * a.ph + j) * a.W + w * a.pw + u;
  const float v = a.latent_f32 ? static_cast<const float*>(a.latent)[src]
                               : __bfloat162float(static_cast<const __nv_bfloat16*>(a.latent)[src]);
  const __nv_bfloat16 bv = __float2bfloat16_rn(v);
  for (int b = 0; b < a.batch; ++b) a.out[((int64_t)b * L + l) * a.K + k] = bv;
}

int patchify(const wanb200_patchify_params* p, cudaStream_t st) {
  if (!p || !p->latent || !p->out) return set_error(WANB200_EINVAL, "patchify: null latent / out");
  if (p->channels <= 0 || p->frames <= 0 || p->height <= 0 || p->width <= 0 || p->pf <= 0 || p->ph <= 0 ||
      p->pw <= 0 || p->batch <= 0 || p->frames % p->pf || p->height % p->ph || p->width % p->pw)
    return set_error(WANB200_EINVAL, "patchify: positive sizes with frames / height / width divisible by the patch");
  if (p->channels * p->frames * p->height * p->width > INT32_MAX || p->batch > 64)
    return set_error(WANB200_EINVAL, "patchify: latent too large (< 2^31 elements, batch <= 64)");
  PatchArgs a;
  a.latent = p->latent;
  a.latent_f32 = p->latent_f32 != 0;
  a.C = (int)p->channels;
  a.F = (int)p->frames;
  a.H = (int)p->height;
  a.W = (int)p->width;
  a.pf = p->pf;
  a.ph = p->ph;
  a.pw = p->pw;
  a.Fg = a.F / a.pf;
  a.Hg = a.H / a.ph;
  a.Wg = a.W / a.pw;
  a.K = a.C * a.pf * a.ph * a.pw;
  a.batch = (int)p->batch;
  a.out = static_cast<__nv_bfloat16*>(p->out);
  const int64_t n = (int64_t)a.Fg * a.Hg * a.Wg * a.K;
  patchify_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("patchify_kernel launch", e);
  return WANB200_OK;
}

struct UnpatchArgs {
  const float* y;  // [batch, L, pf*ph*pw*C]
  int batch, C, Fg, Hg, Wg, pf, ph, pw;
  int mode;
  float guide;
  void* out;  // [C, Fg*pf, Hg*ph, Wg*pw]
  int out_f32;
};

// Thread = one output element (c, fo, ho, wo).  The head's output row of token (f, h, w) holds
// the patch as (i, j, u, c) (`y.view(B, f, h, w, p, q, r, c).permute(0, 7, 1, 4, 2, 5, 3, 6)`,
// fast_dit.py:500-502); the CFG branches combine as uncond + g * (cond - uncond) (503-505), or a
// CFG-parallel rank scales its single branch by its weight (522-523).
__global__ void __launch_bounds__(256) unpatchify_cfg_kernel(const UnpatchArgs a) {
  const int FO = a.Fg * a.pf, HO = a.Hg * a.ph, WO = a.Wg * a.pw;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)a.C * FO * HO * WO) return;
  const int wo = (int)(idx % WO), ho = (int)((idx / WO) % HO), fo = (int)((idx / ((int64_t)WO * HO)) % FO);
  const int c = (int)(idx / ((int64_t)WO * HO * FO));
  const int f = fo / a.pf, i = fo % a.pf, h = ho / a.ph, j = ho % a.ph, w = wo / a.pw, u = wo % a.pw;
  const int64_t L = (int64_t)a.Fg * a.Hg * a.Wg;
  const int64_t l = ((int64_t)f * a.Hg + h) * a.Wg + w;
  const int Kc = a.pf * a.ph * a.pw * a.C;
  const int64_t k = (((int64_t)i * a.ph + j) * a.pw + u) * a.C + c;
  float v;
  if (a.mode == WANB200_CFG_COMBINE) {
    const float cond = a.y[l * Kc + k], uncond = a.y[(L + l) * Kc + k];
    v = uncond + a.guide * (cond - uncond);
  } else {
    v = a.guide * a.y[l * Kc + k];
  }
  if (a.out_f32)
    static_cast<float*>(a.out)[idx] = v;
  else
    static_cast<__nv_bfloat16*>(a.out)[idx] = __float2bfloat16_rn(v);
}

int unpatchify_cfg(const wanb200_unpatchify_params* p, cudaStream_t st) {
  if (!p || !p->y || !p->out) return set_error(WANB200_EINVAL, "unpatchify: null y / out");
  if (p->frames <= 0 || p->height <= 0 || p->width <= 0 || p->pf <= 0 || p->ph <= 0 || p->pw <= 0 ||
      p->channels <= 0)
    return set_error(WANB200_EINVAL, "unpatchify: sizes must be positive");
  if (p->mode != WANB200_CFG_COMBINE && p->mode != WANB200_CFG_SCALE)
    return set_error(WANB200_EINVAL, "unpatchify: mode must be WANB200_CFG_COMBINE or WANB200_CFG_SCALE");
  if (p->mode == WANB200_CFG_COMBINE && p->batch != 2)
    return set_error(WANB200_EINVAL, "unpatchify: the CFG combine needs batch 2 (cond, uncond)");
  if (p->mode == WANB200_CFG_SCALE && p->batch < 1) return set_error(WANB200_EINVAL, "unpatchify: batch >= 1");
  const int64_t n = p->channels * p->frames * p->pf * p->height * p->ph * p->width * p->pw;
  if (n > INT32_MAX || p->batch * n > INT32_MAX) return set_error(WANB200_EINVAL, "unpatchify: too large");
  UnpatchArgs a;
  a.y = p->y;
  a.batch = (int)p->batch;
  a.C = (int)p->channels;
  a.Fg = (int)p->frames;
  a.Hg = (int)p->height;
  a.Wg = (int)p->width;
  a.pf = p->pf;
  a.ph = p->ph;
  a.pw = p->pw;
  a.mode = p->mode;
  a.guide = p->guide;
  a.out = p->out;
  a.out_f32 = p->out_f32 != 0;
  unpatchify_cfg_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("unpatchify_cfg_kernel launch", e);
  return WANB200_OK;
}

}  // namespace wanb200

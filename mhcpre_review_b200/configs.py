"""Synthetic workloads of the benchmark configurations (seeded, reproducible).

The five configurations are the operator's headline benchmark cases:
  c1  CPU-checkable case: M=64 (B=1,S=64), n=4, D=256, fp16, phi~N(0,0.02), no gamma,
      alpha=1, bias~N(0,0.1)
  c2  M=4096 (B=2,S=2048), n=4, D=2560, bf16, phi~N(0,0.01), gamma~1+N(0,0.05)
  c3  M=16384 (B=4,S=4096), n=8, D=4096, bf16 with 1% of x scaled by 20,
      phi~N(0,0.005), no gamma
  c4  M=65536 (B=16,S=4096), n=4, D=7168, bf16, phi~N(0,0.005), gamma~1+N(0,0.05)
  c5  decode sweep M in {1,8,32,128,512} (B=1,S=M), n=4, D=7168, fp16,
      phi~N(0,0.005), gamma on or off
x ~ N(0,1) rounded to the x dtype; alpha ~ U(0.5,1.5) unless fixed; bias ~ N(0,0.1);
normEps = hcEps = 1e-6.  phi is stored [mix][n*D] (K-contiguous), the layout the
reference kernel reads (code/op_kernel/mhc_pre.cpp:535, cloud_runner/runner.cpp:157).

Inputs are generated on the target device with torch's Philox generator seeded
from (seed, tensor id), so a config is the same bytes on every run.
"""
from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class Config:
    name: str
    batch: int
    seq: int
    n: int
    D: int
    dtype: str          # "fp16" | "bf16"
    phi_std: float
    gamma: bool
    alpha_fixed: float | None = None   # None: alpha ~ U(0.5, 1.5)
    outlier_frac: float = 0.0
    outlier_scale: float = 1.0
    seed: int = 0
    norm_eps: float = 1e-6
    hc_eps: float = 1e-6

    @property
    def M(self) -> int:
        return self.batch * self.seq

    @property
    def K(self) -> int:
        return self.n * self.D

    @property
    def mix(self) -> int:
        return self.n * self.n + 2 * self.n

    def algorithmic_bytes(self) -> int:
        """x + hIn (16-bit) + hPost + hRes + phi + gamma + bias + alpha, each once."""
        s = 2
        b = (self.M * self.K * s + self.M * self.D * s + 4 * self.M * self.n + 4 * self.M * self.n * self.n
             + 4 * self.K * self.mix + 4 * self.mix + 12)
        if self.gamma:
            b += 4 * self.K
        return b

    def algorithmic_flops(self) -> int:
        return 2 * self.M * self.K * self.mix


CONFIGS = {
    "c1": Config("c1", 1, 64, 4, 256, "fp16", 0.02, False, alpha_fixed=1.0),
    "c2": Config("c2", 2, 2048, 4, 2560, "bf16", 0.01, True),
    "c3": Config("c3", 4, 4096, 8, 4096, "bf16", 0.005, False, outlier_frac=0.01, outlier_scale=20.0),
    "c4": Config("c4", 16, 4096, 4, 7168, "bf16", 0.005, True),
}
for _m in (1, 8, 32, 128, 512):
    for _g in (True, False):
        _name = f"c5_m{_m}_{'g' if _g else 'ng'}"
        CONFIGS[_name] = Config(_name, 1, _m, 4, 7168, "fp16", 0.005, _g)


def with_shape(cfg: Config, **kw) -> Config:
    return replace(cfg, **kw)


def make_inputs(cfg: Config, device="cuda"):
    """Returns dict x [B,S,n,D], phi [mix,K], alpha [3], bias [mix], gamma [n,D] or None."""
    import torch

    dt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float16

    def gen(tid):
        g = torch.Generator(device=device)
        g.manual_seed(cfg.seed * 1000003 + tid)
        return g

    x = torch.randn((cfg.batch, cfg.seq, cfg.n, cfg.D), generator=gen(1), device=device, dtype=dt)
    if cfg.outlier_frac > 0:
        mask = torch.rand((cfg.batch, cfg.seq, cfg.n, cfg.D), generator=gen(6), device=device) < cfg.outlier_frac
        x = torch.where(mask, x * cfg.outlier_scale, x)
    phi = torch.randn((cfg.mix, cfg.K), generator=gen(2), device=device, dtype=torch.float32) * cfg.phi_std
    gamma = None
    if cfg.gamma:
        gamma = 1.0 + 0.05 * torch.randn((cfg.n, cfg.D), generator=gen(3), device=device, dtype=torch.float32)
    bias = 0.1 * torch.randn((cfg.mix,), generator=gen(4), device=device, dtype=torch.float32)
    if cfg.alpha_fixed is not None:
        alpha = torch.full((3,), cfg.alpha_fixed, device=device, dtype=torch.float32)
    else:
        alpha = 0.5 + torch.rand((3,), generator=gen(5), device=device, dtype=torch.float32)
    return {"x": x.contiguous(), "phi": phi.contiguous(), "alpha": alpha, "bias": bias, "gamma": gamma}

"""CPU oracle for the BoaConstrictor byte predictor (step and full-sequence).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of ``bench.py`` as the checker / timed CPU baseline.  The
product path never imports it.

It restates, in plain torch on a state_dict, the model the reference builds
(paths relative to the reference project root):

* ``BoaBytePredictor`` ``model.py:83-131``: embedding -> L blocks -> head
  Linear(d,d) -> ReLU -> Linear(d,vocab) (``model.py:90-95``).
* ``MambaBlock.forward`` ``model.py:57-65``: ``x + ff(ln2(mamba(ln1(x))))`` with
  LayerNorm eps 1e-5 and ff = Linear(d,4d) -> exact-erf GELU -> Linear(4d,d)
  (``model.py:45-56``).
* The Mamba mixer step (third-party ``mamba_ssm.Mamba.step``, whose op order is
  also spelled out in ``portability_solved_cpp/boa_gpu.hpp:188-218`` and
  ``portability_solved_cpp/mamba_kernels.cu:158-192,264-338``):
  in_proj -> split x,z -> depthwise causal conv (width 4) state shift -> SiLU ->
  x_proj -> split dt,B,C -> dt_proj (+bias) -> softplus -> dA = exp(dt*A),
  A = -exp(A_log) -> h = dA*h + dt*B*x -> y = C.h + D*x -> y*SiLU(z) -> out_proj.

``softplus`` follows torch.nn.functional.softplus (threshold 20), which is what
``mamba_ssm`` applies (``dt_softplus=True``).

State per layer: ``conv`` [B, E, 3] (the last three conv inputs, oldest first)
and ``ssm`` [B, E, N].
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class OracleConfig:
    d_model: int
    n_layers: int
    vocab: int = 256
    d_state: int = 16
    d_conv: int = 4
    expand: int = 2

    @property
    def d_inner(self) -> int:
        return self.expand * self.d_model

    @property
    def dt_rank(self) -> int:
        return math.ceil(self.d_model / 16)


def config_from_state_dict(sd) -> OracleConfig:
    vocab, d = sd["embedding.weight"].shape
    n = 0
    while f"blocks.{n}.ln1.weight" in sd:
        n += 1
    return OracleConfig(d_model=d, n_layers=n, vocab=vocab)


def _ln(x, w, b):
    return F.layer_norm(x, (x.shape[-1],), w, b, 1e-5)


def init_state(cfg: OracleConfig, batch: int, dtype=torch.float32):
    E, N = cfg.d_inner, cfg.d_state
    return [(torch.zeros(batch, E, cfg.d_conv - 1, dtype=dtype),
             torch.zeros(batch, E, N, dtype=dtype)) for _ in range(cfg.n_layers)]


def _mixer_step(sd, p, cfg: OracleConfig, u, conv, ssm):
    E, R, N = cfg.d_inner, cfg.dt_rank, cfg.d_state
    dt_ = u.dtype
    xz = u @ sd[p + "in_proj.weight"].to(dt_).T
    x, z = xz[:, :E], xz[:, E:]
    w = sd[p + "conv1d.weight"].to(dt_).reshape(E, cfg.d_conv)
    window = torch.cat([conv, x.unsqueeze(-1)], dim=-1)          # [B, E, 4]
    xc = (window * w).sum(-1) + sd[p + "conv1d.bias"].to(dt_)
    xc = F.silu(xc)
    new_conv = window[:, :, 1:]
    dbc = xc @ sd[p + "x_proj.weight"].to(dt_).T
    dtr, Bm, Cm = dbc[:, :R], dbc[:, R:R + N], dbc[:, R + N:R + 2 * N]
    dt = dtr @ sd[p + "dt_proj.weight"].to(dt_).T + sd[p + "dt_proj.bias"].to(dt_)
    dt = F.softplus(dt)
    A = -torch.exp(sd[p + "A_log"].to(dt_))                      # [E, N]
    dA = torch.exp(dt.unsqueeze(-1) * A)                          # [B, E, N]
    dBx = dt.unsqueeze(-1) * Bm.unsqueeze(1) * xc.unsqueeze(-1)
    new_ssm = ssm * dA + dBx
    y = (new_ssm * Cm.unsqueeze(1)).sum(-1) + sd[p + "D"].to(dt_) * xc
    y = y * F.silu(z)
    out = y @ sd[p + "out_proj.weight"].to(dt_).T
    return out, new_conv, new_ssm


@torch.inference_mode()
def step(sd, cfg: OracleConfig, tokens: torch.Tensor, state, dtype=torch.float32):
    """One byte for every stream: tokens [B] int64 -> logits [B, vocab]."""
    h = sd["embedding.weight"].to(dtype)[tokens.long()]
    new_state = []
    for i in range(cfg.n_layers):
        p = f"blocks.{i}."
        u = _ln(h, sd[p + "ln1.weight"].to(dtype), sd[p + "ln1.bias"].to(dtype))
        conv, ssm = state[i]
        o, conv, ssm = _mixer_step(sd, p + "mamba.", cfg, u, conv, ssm)
        new_state.append((conv, ssm))
        v = _ln(o, sd[p + "ln2.weight"].to(dtype), sd[p + "ln2.bias"].to(dtype))
        f = F.gelu(v @ sd[p + "ff.0.weight"].to(dtype).T + sd[p + "ff.0.bias"].to(dtype))
        h = h + f @ sd[p + "ff.2.weight"].to(dtype).T + sd[p + "ff.2.bias"].to(dtype)
    r = torch.relu(h @ sd["head.0.weight"].to(dtype).T + sd["head.0.bias"].to(dtype))
    logits = r @ sd["head.2.weight"].to(dtype).T + sd["head.2.bias"].to(dtype)
    return logits, new_state


@torch.inference_mode()
def forward(sd, cfg: OracleConfig, x: torch.Tensor, dtype=torch.float32):
    """Full sequence x [B, L] -> logits [B, L, vocab] by a sequential scan.

    Equals ``model.py:97-101`` for a model whose Mamba layers start from a zero
    state; written as a loop over ``step`` so the two can never disagree.
    """
    B, L = x.shape
    st = init_state(cfg, B, dtype)
    outs = []
    for t in range(L):
        lg, st = step(sd, cfg, x[:, t], st, dtype)
        outs.append(lg)
    return torch.stack(outs, dim=1)


def softmax_probs(logits: torch.Tensor) -> torch.Tensor:
    """What the reference codec feeds the coder: ``codec.py:66,134``."""
    return torch.softmax(logits, dim=-1).to(torch.float32)

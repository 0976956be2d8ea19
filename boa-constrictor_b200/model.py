"""Drop-in for the reference ``model.py``: ``BoaConstrictor(d_model, num_layers,
vocab_size, device)`` returns a ``BoaBytePredictor`` with the reference's module
tree and state_dict keys (model.py:42-134, the key set that
portability_solved_cpp/convert_boa_weights.py:16-135 reads).

The Mamba mixer is this build's own module with mamba_ssm's parameter shapes
and initialisation recipe (mamba_ssm itself is not a dependency): d_state 16,
d_conv 4, expand 2, dt_rank ceil(d_model/16), in_proj/out_proj without bias,
dt_proj weight U(+-dt_rank^-0.5), dt_proj bias = softplus^-1 of a log-uniform
dt in [1e-3, 1e-1] floored at 1e-4, A_log = log(1..16), D = 1.

Inference (``init_stream`` / ``step`` / ``forward``) runs on the sm_100a kernel
in libboa_b200.so (``boa_model_step`` / ``boa_model_logits``) on a CUDA
device; there is no CPU execution path.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.nn as nn

from boa_b200 import _native as _n
from boa_b200.weights import flatten_state_dict

D_STATE = 16
D_CONV = 4
EXPAND = 2

# Projection operand formats of the kernel.  "tf32x3" (the default) splits every
# fp32 weight and activation into tf32 hi + lo halves whose products are summed
# in fp32: the arithmetic of the reference's fp32 nn.Linear to within fp32
# rounding.  "f16x2" carries the same 22 significant bits as an fp16 hi and an
# fp16 residual scaled by 2^11, at half the weight bytes, for activations
# below 65504 in magnitude (larger ones are reported, BOA_ERR_RANGE).  "tf32",
# "fp16" and "bf16" are faster, narrower alternatives ("bf16" is what the
# d_model-512 configuration specifies).
WEIGHT_FORMATS = {"tf32x3": _n.BOA_WEIGHTS_TF32X3, "f16x2": _n.BOA_WEIGHTS_F16X2, "tf32": _n.BOA_WEIGHTS_TF32,
                  "bf16": _n.BOA_WEIGHTS_BF16, "fp16": _n.BOA_WEIGHTS_F16}


def default_format(d_model: int) -> str:
    """The operand kind used when none is given: "f16x2" (fp32-equivalent; its
    probabilities at d_model 256 / 8 layers are within 1.5e-8 of an fp64
    evaluation, the reference's own fp32 arithmetic within 6e-9) for
    d_model <= 256, and "bf16" for d_model 512, where the split kinds do not
    fit shared memory and TMEM (the d_model-512 configuration specifies bf16)."""
    return "f16x2" if d_model <= 256 else "bf16"


class Mamba(nn.Module):
    """Parameters of one Mamba mixer (shapes and init as mamba_ssm.Mamba(d_model))."""

    def __init__(self, d_model: int, dt_min: float = 1e-3, dt_max: float = 1e-1, dt_init_floor: float = 1e-4):
        super().__init__()
        self.d_model = d_model
        self.d_state = D_STATE
        self.d_conv = D_CONV
        self.d_inner = EXPAND * d_model
        self.dt_rank = math.ceil(d_model / 16)
        E, R = self.d_inner, self.dt_rank
        self.in_proj = nn.Linear(d_model, 2 * E, bias=False)
        self.conv1d = nn.Conv1d(E, E, kernel_size=D_CONV, groups=E, padding=D_CONV - 1, bias=True)
        self.x_proj = nn.Linear(E, R + 2 * D_STATE, bias=False)
        self.dt_proj = nn.Linear(R, E, bias=True)
        std = R ** -0.5
        with torch.no_grad():
            nn.init.uniform_(self.dt_proj.weight, -std, std)
            dt = torch.exp(torch.rand(E) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
            dt = dt.clamp(min=dt_init_floor)
            self.dt_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))
        A = torch.arange(1, D_STATE + 1, dtype=torch.float32).repeat(E, 1)
        self.A_log = nn.Parameter(torch.log(A))
        self.D = nn.Parameter(torch.ones(E))
        self.out_proj = nn.Linear(E, d_model, bias=False)


class MambaBlock(nn.Module):
    """ln1 -> mamba -> ln2 -> ff -> + x (model.py:42-65)."""

    def __init__(self, d_model: int):
        super().__init__()
        self.ln1 = nn.LayerNorm(d_model)
        self.mamba = Mamba(d_model)
        self.ln2 = nn.LayerNorm(d_model)
        self.ff = nn.Sequential(nn.Linear(d_model, 4 * d_model), nn.GELU(), nn.Linear(4 * d_model, d_model))


class StreamState:
    """Per-stream recurrent state for ``step`` (replaces mamba_ssm's
    InferenceParams, model.py:104-106): conv windows + SSM states of every
    layer, resident on the device in the layout the kernel expects."""

    def __init__(self, model: "BoaBytePredictor", batch_size: int, device):
        self.batch_size = int(batch_size)
        self.device = torch.device(device)
        nb = model._native_handle(self.device).workspace_bytes(self.batch_size)
        self.workspace = torch.zeros(nb, dtype=torch.uint8, device=self.device)
        self.seqlen_offset = 0


class NativeModel:
    """Owns a boa_model handle built from a state_dict snapshot."""

    def __init__(self, sd, d_model: int, n_layers: int, vocab: int, weight_format: int, device_index: int):
        flat = flatten_state_dict(sd)
        h = ctypes.c_void_p()
        _n.call("boa_model_create", ctypes.byref(h), int(d_model), int(n_layers), int(vocab),
                flat.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(flat.size), int(weight_format),
                int(device_index))
        self.h = h
        self.device_index = device_index
        self.d_model, self.n_layers, self.vocab, self.weight_format = d_model, n_layers, vocab, weight_format

    def workspace_bytes(self, n: int) -> int:
        return int(_n.load().boa_model_workspace_bytes(self.h, int(n)))

    def set_time_block(self, positions: int) -> None:
        """Positions per kernel step for encode / logits runs: 0 (default: each
        launch chooses 4 or 8), 1, 4 or 8.  The output bits are the same."""
        _n.call("boa_model_set_time_block", self.h, int(positions))

    def time_block(self, n_chunks: int, positions: int) -> int:
        """Positions per kernel step an encode / logits launch of this shape takes."""
        tb = ctypes.c_int(0)
        _n.call("boa_model_time_block", self.h, int(n_chunks), int(positions), ctypes.byref(tb))
        return tb.value

    def check(self, stream=None) -> None:
        """Wait for `stream` (torch's current stream by default) and raise the
        device-side errors of this model's calls enqueued so far
        (boa_model_status: timeouts, overflowing streams, bad symbols)."""
        import torch
        if stream is None:
            stream = torch.cuda.current_stream(torch.device("cuda", self.device_index))
        _n.call("boa_model_status", self.h, ctypes.c_void_p(int(stream.cuda_stream)))

    def tile_bytes_per_step(self) -> int:
        v = ctypes.c_size_t()
        _n.call("boa_model_info", self.h, None, None, None, None, ctypes.byref(v))
        return int(v.value)

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            _n.load().boa_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BoaBytePredictor(nn.Module):
    """Mamba model predicting the next byte (model.py:83-131)."""

    def __init__(self, d_model=256, num_layers=4, vocab_size=256, weight_format: str | None = None):
        super().__init__()
        self.embedding = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([MambaBlock(d_model) for _ in range(num_layers)])
        self.head = nn.Sequential(nn.Linear(d_model, d_model), nn.ReLU(), nn.Linear(d_model, vocab_size))
        self.d_model = d_model
        self.num_layers = num_layers
        self.vocab_size = vocab_size
        self.weight_format = weight_format or default_format(d_model)
        if self.weight_format not in WEIGHT_FORMATS:
            raise ValueError(f"unknown weight_format {weight_format!r}; one of {sorted(WEIGHT_FORMATS)}")
        self._native = {}

    # -- native handle management ---------------------------------------------
    def _param_key(self):
        return tuple((id(p), p._version) for p in self.parameters()), self.weight_format

    def _native_handle(self, device) -> NativeModel:
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("boa_b200 inference runs on CUDA devices only (no CPU path)")
        _n.require_cuda()
        idx = device.index if device.index is not None else torch.cuda.current_device()
        key = (idx,) + self._param_key()
        nm = self._native.get(idx)
        if nm is None or nm[0] != key:
            sd = {k: v.detach().float().cpu() for k, v in self.state_dict().items()}
            self._native[idx] = (key, NativeModel(sd, self.d_model, self.num_layers, self.vocab_size,
                                                  WEIGHT_FORMATS[self.weight_format], idx))
        return self._native[idx][1]

    def native(self, device=None) -> NativeModel:
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        return self._native_handle(device)

    # -- reference API ----------------------------------------------------------
    @torch.inference_mode()
    def init_stream(self, max_len: int, batch_size: int = 1, device=None, dtype=None):
        if device is None:
            device = "cuda"
        return StreamState(self, batch_size, device)

    @torch.inference_mode()
    def step(self, byte_t: torch.LongTensor, inf: StreamState) -> torch.Tensor:
        """byte_t [B] -> logits [B, vocab] (model.py:108-117)."""
        dev = inf.device
        nm = self._native_handle(dev)
        toks = byte_t.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
        B = toks.numel()
        if B != inf.batch_size:
            raise ValueError(f"step got {B} tokens for a stream of batch {inf.batch_size}")
        out = torch.empty((B, self.vocab_size), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _n.call("boa_model_step", nm.h, B, ctypes.c_void_p(toks.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                    ctypes.c_void_p(inf.workspace.data_ptr()), ctypes.c_size_t(inf.workspace.numel()),
                    ctypes.c_void_p(_n.stream_ptr(dev)))
        inf.seqlen_offset += 1
        return out

    @torch.inference_mode()
    def forward(self, x, inference_params=None):
        """x [B, L] -> logits [B, L, vocab] from a zero state (model.py:97-101)."""
        dev = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
        nm = self._native_handle(dev)
        B, L = x.shape
        toks = x.to(device=dev, dtype=torch.int32).contiguous()
        out = torch.empty((B, L, self.vocab_size), dtype=torch.float32, device=dev)
        ws = torch.empty(nm.workspace_bytes(B), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            _n.call("boa_model_logits", nm.h, B, L, ctypes.c_void_p(toks.data_ptr()),
                    ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                    ctypes.c_size_t(ws.numel()), ctypes.c_void_p(_n.stream_ptr(dev)))
        return out


def BoaConstrictor(d_model=256, num_layers=4, vocab_size=256, device="cuda", weight_format: str | None = None):
    """Construct a BoaBytePredictor (model.py:5-134).  Parameters are created on
    the CPU with the module-construction order of the reference (embedding,
    blocks, head) so a given torch seed always yields the same weights; the
    codec moves nothing to the GPU but the packed kernel weights."""
    model = BoaBytePredictor(d_model=d_model, num_layers=num_layers, vocab_size=vocab_size,
                             weight_format=weight_format)
    i = 0
    for m in model.modules():
        if isinstance(m, Mamba):
            m.layer_idx = i
            i += 1
    return model


def seeded_model(d_model: int, num_layers: int, vocab_size: int = 256, seed: int = 0,
                 weight_format: str | None = None) -> BoaBytePredictor:
    """The benchmark/test model: torch.manual_seed(seed) then construction."""
    torch.manual_seed(seed)
    return BoaConstrictor(d_model=d_model, num_layers=num_layers, vocab_size=vocab_size, device="cpu",
                          weight_format=weight_format)

"""Muon / NorMuon / Hyperball optimizers with auxiliary Adam (reference: koochak/optim/muon.py:13-573).

Semantics follow the reference exactly (momentum lerp, Nesterov, quintic
Newton-Schulz with (a, b, c) = (3.4445, -4.7750, 2.0315) in bf16 after
Frobenius normalisation, Moonlight scale 0.2*sqrt(max(rows, cols)), decoupled
weight decay; bias-corrected Adam for the aux groups; per-parameter state
``momentum_buffer`` / ``exp_avg``, ``exp_avg_sq`` and an int ``step``), so
optimizer state dicts are interchangeable with the reference's.

Execution:

* CPU or non-fp32 parameters run the plain-PyTorch functions below (they are
  also the oracle of the tests).
* CUDA fp32 parameters run the native path. Muon matrices are bucketed by
  shape, and buckets whose shapes differ only by a transpose share one
  Newton-Schulz batch; per bucket one kernel applies the clip coefficient, momentum and
  Nesterov and writes bf16 (transposed when rows > cols) while accumulating
  the Frobenius norms, one kernel normalises, the 5 Newton-Schulz iterations
  are 15 batched tcgen05 GEMMs with the ``b*A + c*A@A`` and ``a*X + B@X``
  combinations fused into their epilogues, and one kernel applies the update
  with weight decay, the EMA of the new parameter and its bf16 copy. Aux Adam
  groups are one multi-tensor kernel (clip coefficient, moments, bias
  correction, decoupled weight decay, EMA and bf16 copy).
* Distributed classes (chosen when a process group exists) shard the Muon
  work: matrix i of the size-sorted group is owned by rank i % world, as in
  the reference (its momentum lives only there). On CUDA the group's matrices are stored in one
  symmetric-memory slab (``parallel.symm.SymmetricParamSlab``) and the
  owner's update kernel stores each new matrix into every rank's copy over
  NVLink (P2P stores, or ``multimem.st`` through NVSwitch), followed by one
  bounded cross-GPU barrier per step: the all-gather is fused into the
  update. ``KOOCHAK_B200_MUON_GATHER=nccl`` (or matrices whose column count
  is not a multiple of 4) selects one NCCL all-gather per shape bucket
  instead, with matrix k of each bucket owned by rank k % world.
  Adam groups run on every rank, as in the reference.

The training loop passes the gradient-clip coefficient as a device scalar
(``optimizer.kb_grad_scale``) so gradients are scaled on read instead of being
rewritten, and may hand over a GPU EMA (``optimizer.kb_ema``) to be fused.
"""

from __future__ import annotations

import contextlib
import math
import os
from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..utils import flags

__all__ = ["zeropower_via_newtonschulz5", "muon_update", "normuon_update", "adam_update", "HyperballOptimizer",
           "Muon", "SingleDeviceMuon", "NorMuon", "SingleDeviceNorMuon", "MuonWithAuxAdam",
           "SingleDeviceMuonWithAuxAdam", "NorMuonWithAuxAdam", "SingleDeviceNorMuonWithAuxAdam", "NS_COEFFS"]

NS_COEFFS = (3.4445, -4.7750, 2.0315)


# ----------------------------------------------------------------------------- reference math


@flags.compile_wrap
def zeropower_via_newtonschulz5(G, steps: int):
    """Quintic Newton-Schulz orthogonalisation in bf16 (approximately U S' V^T)."""

    assert G.ndim >= 2
    a, b, c = NS_COEFFS
    X = G.bfloat16()
    tall = G.size(-2) > G.size(-1)
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * A @ A
        X = a * X + B @ X
    return X.mT if tall else X


@flags.compile_wrap
def muon_update(grad, momentum, beta=0.95, ns_steps=5, nesterov=True):
    momentum.lerp_(grad, 1 - beta)
    update = grad.lerp_(momentum, beta) if nesterov else momentum
    if update.ndim > 2:
        update = update.reshape(len(update), -1)
    rows, cols = update.size(-2), update.size(-1)
    update = zeropower_via_newtonschulz5(update, steps=ns_steps)
    update *= 0.2 * max(rows, cols) ** 0.5
    return update


@flags.compile_wrap
def normuon_update(grad, momentum, second_momentum, beta=0.95, beta2=0.95, ns_steps=5, nesterov=True):
    momentum.lerp_(grad, 1 - beta)
    update = grad.lerp_(momentum, beta) if nesterov else momentum
    if update.ndim > 2:
        update = update.reshape(len(update), -1)
    rows, cols = update.size(-2), update.size(-1)
    update = zeropower_via_newtonschulz5(update, steps=ns_steps).float()
    vnorm = update.norm(dim=(-2, -1), keepdim=True)
    v_mean = torch.mean(update * update, dim=-1, keepdim=True)
    second_momentum.lerp_(v_mean, 1 - beta2)
    update.mul_(1 / second_momentum.sqrt().add_(1e-10))
    vnorm_new = update.norm(dim=(-2, -1), keepdim=True)
    update.mul_(vnorm / vnorm_new.add_(1e-10))
    update *= max(1, rows / cols) ** 0.5
    return update


@flags.compile_wrap
def adam_update(grad, buf1, buf2, step, betas, eps):
    buf1.lerp_(grad, 1 - betas[0])
    buf2.lerp_(grad.square(), 1 - betas[1])
    return (buf1 / (1 - betas[0] ** step)) / ((buf2 / (1 - betas[1] ** step)).sqrt() + eps)


def _profile_ranges_on() -> bool:
    return os.environ.get("KAVEH_PROFILE_RANGES", "").lower() in {"1", "true", "yes", "on"}


@contextlib.contextmanager
def _profile_range(name: str):
    if not _profile_ranges_on():
        yield
        return
    with torch.autograd.profiler.record_function(name):
        yield


_PROJECTIONS = ("sphere", "ball")


class HyperballOptimizer:
    """Wraps an optimizer; after each step, pulls chosen matrices back to their starting Frobenius radius.

    (behaviour of reference koochak/optim/muon.py:106-192)

    Each trainable matrix (``ndim >= 2``) with a non-negligible norm keeps the
    radius ``radius_scale * |p_0|``. ``sphere`` rescales it to exactly that
    radius after every step, ``ball`` only shrinks it back when it grew past
    it. On CUDA fp32 matrices the projection is two native launches for all
    matrices together (``hyperball_project``), which also refresh the models'
    bf16 copies; elsewhere it runs as PyTorch ops.
    """

    def __init__(self, inner: torch.optim.Optimizer, params: Iterable[torch.nn.Parameter], *, eps: float = 1.0e-8,
                 radius_scale: float = 1.0, projection: str = "sphere") -> None:
        kind = str(projection).lower()
        if float(radius_scale) <= 0.0:
            raise ValueError("radius_scale must be positive")
        if kind not in _PROJECTIONS:
            raise ValueError("projection must be 'sphere' or 'ball'")
        self.inner = inner
        self.eps, self.radius_scale, self.projection = float(eps), float(radius_scale), kind
        self.params: List[torch.nn.Parameter] = []
        self.radii: List[torch.Tensor] = []
        for p in dict.fromkeys(params):  # first occurrence of each parameter, in order
            if not (p.requires_grad and p.ndim >= 2):
                continue
            start = p.detach().float().norm()
            if float(start) > self.eps:
                self.params.append(p)
                self.radii.append((start * self.radius_scale).detach())
        self._radius_table: Optional[torch.Tensor] = None

    @property
    def param_groups(self):
        return self.inner.param_groups

    @property
    def state(self):
        return self.inner.state

    def zero_grad(self, *args, **kwargs):
        return self.inner.zero_grad(*args, **kwargs)

    def __getattr__(self, name: str) -> Any:
        if name.startswith("kb_"):
            return getattr(self.inner, name)
        raise AttributeError(name)

    def __setattr__(self, name: str, value: Any) -> None:
        if name.startswith("kb_") and "inner" in self.__dict__:
            setattr(self.inner, name, value)
        else:
            object.__setattr__(self, name, value)

    def _native_projection(self) -> bool:
        if not self.params or not _native_ready(self.params):
            return False
        dev = self.params[0].device
        return all(p.device == dev for p in self.params)

    @torch.no_grad()
    def _project(self) -> None:
        if self._native_projection():
            from ..ops._ext import native

            dev = self.params[0].device
            table = self._radius_table
            if table is None or table.device != dev:
                table = torch.stack([r.to(device=dev, dtype=torch.float32) for r in self.radii])
                self._radius_table = table
            native().hyperball_project(self.params, table, _shadow_list(self.params), self.eps,
                                       self.projection == "ball")
            _mark_shadows(self.params)
            return
        for i, p in enumerate(self.params):
            radius = self.radii[i]
            if radius.device != p.device or radius.dtype != torch.float32:
                radius = self.radii[i] = radius.to(device=p.device, dtype=torch.float32).detach()
            factor = radius / p.detach().float().norm().clamp_min(self.eps)
            if self.projection == "ball":
                factor = torch.minimum(factor, torch.ones_like(factor))
            p.mul_(factor.to(dtype=p.dtype))

    def step(self, closure=None):
        skip = getattr(self.inner, "kb_skip", None)  # read before the inner step consumes it
        with _profile_range("optimizer.hyperball.inner_step"):
            loss = self.inner.step(closure)
        with _profile_range("optimizer.hyperball.project"):
            if skip is not None and not self._native_projection():
                if float(skip.sum()) != 0.0:
                    return loss  # the inner step was skipped: nothing to project
                skip = None
            from ..ops._ext import native

            C = native() if skip is not None else None
            if C is not None:
                C.set_step_skip(skip.float().reshape(-1)[:1].contiguous())
            try:
                self._project()
            finally:
                if C is not None:
                    C.set_step_skip(None)
        return loss

    def state_dict(self) -> dict[str, Any]:
        return {"inner": self.inner.state_dict(),
                "hyperball_radii": [r.detach().cpu().clone() for r in self.radii],
                "hyperball_radius_scale": self.radius_scale, "hyperball_projection": self.projection}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        if "inner" not in state_dict:
            self.inner.load_state_dict(state_dict)
            return
        self.inner.load_state_dict(state_dict["inner"])
        saved = state_dict.get("hyperball_radii")
        if saved is not None and len(saved) == len(self.radii):
            self.radii = [torch.as_tensor(r).detach().clone() for r in saved]
            self._radius_table = None


# ----------------------------------------------------------------------------- reference-path group steps


def _foreach_adam_enabled(group: Dict[str, Any]) -> bool:
    if "foreach_adam_update" in group:
        return bool(group["foreach_adam_update"])
    return os.environ.get("KAVEH_ADAM_FOREACH_UPDATE", "").lower() in {"1", "true", "yes", "on"}


def _ensure_grad(p: torch.nn.Parameter) -> None:
    if p.grad is None:
        p.grad = torch.zeros_like(p)


def _apply_update(p: torch.nn.Parameter, update: torch.Tensor, group: Dict[str, Any]) -> None:
    p.mul_(1 - group["lr"] * group["weight_decay"])
    p.add_(update.reshape(p.shape), alpha=-group["lr"])


def _muon_param_update(p, group, state):
    if "momentum_buffer" not in state:
        state["momentum_buffer"] = torch.zeros_like(p)
    return muon_update(p.grad, state["momentum_buffer"], beta=group["momentum"])


def _normuon_param_update(p, group, state):
    if "momentum_buffer" not in state:
        state["momentum_buffer"] = torch.zeros_like(p)
        shape = (p.shape[0], 1) if p.ndim > 2 else (*p.shape[:-1], 1)
        state["second_momentum_buffer"] = torch.zeros(shape, dtype=p.dtype, device=p.device)
    return normuon_update(p.grad, state["momentum_buffer"], state["second_momentum_buffer"], beta=group["momentum"],
                          beta2=group["beta2"])


def _adam_param_update(p, group, state):
    if "exp_avg" not in state:
        state["exp_avg"] = torch.zeros_like(p)
        state["exp_avg_sq"] = torch.zeros_like(p)
        state["step"] = 0
    state["step"] += 1
    return adam_update(p.grad, state["exp_avg"], state["exp_avg_sq"], state["step"], group["betas"], group["eps"])


def _clip_scale(optimizer) -> Optional[torch.Tensor]:
    return getattr(optimizer, "kb_grad_scale", None)


def _scaled_grad_inplace(optimizer, p) -> None:
    """Reference path: apply a pending clip coefficient to ``p.grad`` in place."""

    s = _clip_scale(optimizer)
    if s is not None and p.grad is not None:
        p.grad.mul_(s.to(device=p.grad.device, dtype=p.grad.dtype))


def _ref_muon_group(optimizer, group, update_fn, distributed: bool) -> None:
    params: List[torch.nn.Parameter] = group["params"]
    if not params:
        return
    if not distributed:
        for p in params:
            _ensure_grad(p)
            _scaled_grad_inplace(optimizer, p)
            _apply_update(p, update_fn(p, group, optimizer.state[p]), group)
        return
    world, rank = dist.get_world_size(), dist.get_rank()
    padded = params + [torch.empty_like(params[-1])] * (world - len(params) % world)
    for base in range(0, len(params), world):
        i = base + rank
        if i < len(params):
            p = params[i]
            _ensure_grad(p)
            _scaled_grad_inplace(optimizer, p)
            _apply_update(p, update_fn(p, group, optimizer.state[p]), group)
        dist.all_gather(padded[base:base + world], padded[base + rank])


def _ref_adam_group(optimizer, group) -> None:
    for p in group["params"]:
        _ensure_grad(p)
        _scaled_grad_inplace(optimizer, p)
    if _foreach_adam_enabled(group) and _foreach_adam_group(optimizer, group):
        return
    for p in group["params"]:
        _apply_update(p, _adam_param_update(p, group, optimizer.state[p]), group)


def _foreach_adam_group(optimizer, group) -> bool:
    params = list(group["params"])
    if not params:
        return True
    if len({p.device for p in params}) != 1 or len({p.dtype for p in params}) != 1:
        return False
    states = []
    for p in params:
        st = optimizer.state[p]
        if "exp_avg" not in st:
            st["exp_avg"] = torch.zeros_like(p)
            st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] = 0
        states.append(st)
    if len({int(st["step"]) for st in states}) != 1:
        return False
    step = int(states[0]["step"]) + 1
    for st in states:
        st["step"] = step
    grads = [p.grad for p in params]
    m = [st["exp_avg"] for st in states]
    v = [st["exp_avg_sq"] for st in states]
    b1, b2 = group["betas"]
    sq_bc2 = (1 - b2 ** step) ** 0.5
    step_size = group["lr"] * sq_bc2 / (1 - b1 ** step)
    torch._foreach_lerp_(m, grads, 1 - b1)
    torch._foreach_lerp_(v, torch._foreach_mul(grads, grads), 1 - b2)
    denom = torch._foreach_sqrt(v)
    torch._foreach_add_(denom, group["eps"] * sq_bc2)
    if float(group["weight_decay"]) != 0.0:
        torch._foreach_mul_(params, 1 - group["lr"] * float(group["weight_decay"]))
    torch._foreach_addcdiv_(params, m, denom, value=-step_size)
    return True


# ----------------------------------------------------------------------------- native path

_EMPTY_CACHE: Dict[torch.device, torch.Tensor] = {}


def _empty(device: torch.device) -> torch.Tensor:
    t = _EMPTY_CACHE.get(device)
    if t is None:
        t = torch.empty(0, device=device, dtype=torch.float32)
        _EMPTY_CACHE[device] = t
    return t


def _native_ready(params: Sequence[torch.Tensor]) -> bool:
    if not params:
        return False
    if not all(p.is_cuda and p.dtype == torch.float32 and p.is_contiguous() for p in params):
        return False
    from ..ops._ext import available

    return available()


def _shadow_list(params: Sequence[torch.Tensor]) -> List[torch.Tensor]:
    """bf16 copies kept by the models (updated in the same pass), or empty placeholders."""

    out = []
    for p in params:
        sh = getattr(p, "_kb_shadow", None)
        ok = sh is not None and sh.shape == p.shape and sh.device == p.device and sh.dtype == torch.bfloat16
        out.append(sh if ok else _empty(p.device))
    return out


def _mark_shadows(params: Sequence[torch.Tensor]) -> None:
    for p in params:
        if getattr(p, "_kb_shadow", None) is not None and p._kb_shadow.dtype == torch.bfloat16:  # type: ignore
            p._kb_shadow_version = p._version  # type: ignore[attr-defined]


def _ema_list(optimizer, params: Sequence[torch.Tensor]) -> Tuple[List[torch.Tensor], float]:
    fused = getattr(optimizer, "kb_ema", None)
    if not fused:
        return [], 0.0
    d, by_id = fused
    return [by_id.get(id(p), _empty(p.device)) for p in params], float(d)


def _native_adam_group(optimizer, group) -> None:
    from ..ops._ext import native

    params = list(group["params"])
    grads, m, v, steps = [], [], [], []
    for p in params:
        _ensure_grad(p)
        st = optimizer.state[p]
        if "exp_avg" not in st:
            st["exp_avg"] = torch.zeros_like(p)
            st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] = 0
        st["step"] = int(st["step"]) + 1
        g = p.grad
        if g.dtype != torch.float32 or not g.is_contiguous():
            g = g.float().contiguous()
        grads.append(g)
        m.append(st["exp_avg"])
        v.append(st["exp_avg_sq"])
        steps.append(int(st["step"]))
    ema, d = _ema_list(optimizer, params)
    b1, b2 = group["betas"]
    native().adamw_step(params, grads, m, v, steps, ema, _shadow_list(params), _clip_scale(optimizer),
                        float(group["lr"]), float(b1), float(b2), float(group["eps"]), float(group["weight_decay"]), d)
    _mark_shadows(params)


def newton_schulz_batched(X: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """In-place-style NS5 on a normalised bf16 batch [n, r, c] (r <= c) with tcgen05 GEMMs.

    ``X X^T`` and ``b A + c A A`` are symmetric, so those two GEMMs compute
    only the tiles on or above the diagonal and mirror them, where the inner
    dimension is long enough for the saved tiles to outweigh the mirrored
    stores (measured: 1.2-1.7x faster at 2048 x 5504 and 768 x 3072, no gain
    or a loss at 768 x 768).
    """

    from ..ops import functional as kf

    a, b, c = NS_COEFFS
    n, r, cols = X.shape
    A = torch.empty((n, r, r), device=X.device, dtype=torch.bfloat16)
    B = torch.empty_like(A)
    Y = torch.empty_like(X)
    sym_xx, sym_aa = cols >= 1536, r >= 1024
    for _ in range(steps):
        kf.gemm(X, X, out=A, symmetric=sym_xx)                   # A = X X^T
        kf.gemm(A, A, out=B, d=A, alpha=c, beta=b, symmetric=sym_aa)  # B = b A + c A A   (A symmetric)
        kf.gemm(B, X, b_mn_major=True, out=Y, d=X, beta=a)   # X' = a X + B X
        X, Y = Y, X
    return X


def _muon_buckets(params: Sequence[torch.nn.Parameter]) -> Dict[Tuple[int, int], List[int]]:
    buckets: Dict[Tuple[int, int], List[int]] = {}
    for i, p in enumerate(params):
        R = p.shape[0]
        C = p.numel() // R
        buckets.setdefault((R, C), []).append(i)
    return buckets


def _native_muon_bucket(optimizer, group, parts: List[Tuple[int, int, List[torch.nn.Parameter]]],
                        slab=None) -> None:
    """Muon (or NorMuon) on matrices that orthogonalise as one batch.

    ``parts`` lists (R, C, params) groups whose shapes agree up to a
    transpose (all [R, C] or [C, R]): the prologue writes each matrix in its
    wide orientation [min, max] into one bf16 batch, Newton-Schulz runs once
    over the whole batch (fewer, fuller GEMM launches), and each part's
    epilogue transposes back as needed. For NorMuon each part's per-row
    second moments and update scales come from ``normuon_row_scale`` and the
    update kernels apply one scale per row instead of Muon's scalar.
    """

    from ..ops._ext import native

    normuon = bool(getattr(optimizer, "_normuon", False))
    n = sum(len(ps) for _, _, ps in parts)
    dev = parts[0][2][0].device
    r, c = min(parts[0][0], parts[0][1]), max(parts[0][0], parts[0][1])
    X = torch.empty((n, r, c), device=dev, dtype=torch.bfloat16)
    ss = torch.empty(n, device=dev, dtype=torch.float32)
    base = 0
    for R, C, params in parts:
        grads, moms = [], []
        for p in params:
            _ensure_grad(p)
            st = optimizer.state[p]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros_like(p)
            if normuon and "second_momentum_buffer" not in st:
                st["second_momentum_buffer"] = torch.zeros((p.shape[0], 1), dtype=p.dtype, device=p.device)
            g = p.grad
            if g.dtype != torch.float32 or not g.is_contiguous():
                g = g.float().contiguous()
            grads.append(g)
            moms.append(st["momentum_buffer"])
        k = len(params)
        native().muon_prologue(grads, moms, X[base:base + k], ss[base:base + k], _clip_scale(optimizer),
                               float(group["momentum"]), True, R > C)
        base += k
    native().muon_scale(X, ss, n)
    X = newton_schulz_batched(X, 5)
    base = 0
    for R, C, params in parts:
        k = len(params)
        Xi = X[base:base + k]
        base += k
        row_scale = None
        if normuon:
            row_scale = torch.empty((k, R), device=dev, dtype=torch.float32)
            rowsq = torch.empty((k, R), device=dev, dtype=torch.float32)
            native().normuon_row_scale(Xi, R, C, R > C,
                                       [optimizer.state[p]["second_momentum_buffer"].view(-1) for p in params],
                                       float(group["beta2"]), rowsq, row_scale)
        scale = 0.2 * math.sqrt(max(R, C))
        if slab is not None:
            ws = slab.ws
            native().muon_update_gather(params, Xi, _shadow_list(params), float(group["lr"]),
                                        float(group["weight_decay"]), scale, R > C, ws.bases, ws.mc_base, ws.rank,
                                        ws.nbytes, row_scale)
        else:
            ema, d = _ema_list(optimizer, params)
            native().muon_epilogue(params, Xi, ema, _shadow_list(params), float(group["lr"]),
                                   float(group["weight_decay"]), scale, R > C, d, row_scale)
        _mark_shadows(params)


def _batches(owned: Dict[Tuple[int, int], List[torch.nn.Parameter]]
             ) -> List[List[Tuple[int, int, List[torch.nn.Parameter]]]]:
    """Join shape buckets that differ only by a transpose into one Newton-Schulz batch."""

    joined: Dict[Tuple[int, int], List[Tuple[int, int, List[torch.nn.Parameter]]]] = {}
    for (R, C), ps in owned.items():
        if ps:
            joined.setdefault((min(R, C), max(R, C)), []).append((R, C, ps))
    return list(joined.values())


def _slab_ok(params: Sequence[torch.Tensor]) -> bool:
    """Whether the symmetric-slab (in-kernel peer store) path can hold these parameters."""

    if os.environ.get("KOOCHAK_B200_MUON_GATHER", "peer") != "peer":
        return False
    if not dist.is_initialized() or dist.get_backend() != "nccl" or dist.get_world_size() > 8:
        return False
    return _native_ready(params)


def _muon_path(group: Dict[str, Any], normuon: bool, distributed: bool) -> str:
    """How a Muon group is stepped: 'ref' (PyTorch ops), 'native', 'slab' (native + peer stores) or 'nccl'."""

    params = list(group["params"])
    if not _native_ready(params) or any(p.dim() < 2 for p in params):
        return "ref"
    if not distributed:
        return "native"
    if _slab_ok(params) and all(p.dim() >= 2 and (p.numel() // p.shape[0]) % 4 == 0 for p in params):
        return "slab"
    return "nccl"


def muon_owners(group: Dict[str, Any], path: str, world: int) -> List[int]:
    """Owner rank of each parameter of a distributed Muon group (its momentum lives only there).

    Matrix i of the size-sorted group belongs to rank i % W, the reference's
    rule (its distributed step updates ``params[base + rank]``), for the
    PyTorch and slab paths; the NCCL all-gather fallback, which gathers per
    shape bucket, owns matrix k of each bucket on rank k % W.
    """

    params = list(group["params"])
    if path != "nccl":
        return [i % world for i in range(len(params))]
    owners = [0] * len(params)
    for idx in _muon_buckets(params).values():
        for k, i in enumerate(idx):
            owners[i] = k % world
    return owners


def _side_streams(optimizer, device: torch.device, n: int) -> List[torch.cuda.Stream]:
    """``n`` CUDA streams kept on the optimizer for its concurrent Newton-Schulz batches."""

    pool = getattr(optimizer, "_kb_side_streams", None)
    if pool is None:
        pool = []
        optimizer._kb_side_streams = pool
    while len(pool) < n:
        pool.append(torch.cuda.Stream(device=device))
    return pool[:n]


def _native_muon_group(optimizer, group, path: str, slab=None) -> None:
    params: List[torch.nn.Parameter] = list(group["params"])
    if not params:
        return
    buckets = _muon_buckets(params)
    if path == "native":
        batches = _batches({key: [params[i] for i in idx] for key, idx in buckets.items()})
        # One process: the batches are independent, so small ones run on streams of their own. Their
        # Newton-Schulz GEMMs are short (GPT-2: 12 x 768 x 768 is 108 tiles on 74 SM pairs, about 10 us of
        # launch, pipeline fill and tail each), and side by side one batch's gaps are filled by another's
        # tiles. Batches of 2048-row matrices (Llama-style 1.3B) fill the GPU alone and measured 2 % slower
        # side by side, so only batches whose matrices have at most 1024 rows (after the transpose) qualify.
        # (Not across processes: the peer-store update kernels wait on other ranks.)
        small = all(min(parts[0][0], parts[0][1]) <= 1024 for parts in batches)
        if (len(batches) > 1 and small and params[0].is_cuda
                and os.environ.get("KOOCHAK_B200_MUON_STREAMS", "1") != "0"):
            main = torch.cuda.current_stream()
            side = _side_streams(optimizer, params[0].device, len(batches) - 1)
            for st in side:
                st.wait_stream(main)
            for parts, st in zip(batches[1:], side):
                with torch.cuda.stream(st):
                    _native_muon_bucket(optimizer, group, parts)
            _native_muon_bucket(optimizer, group, batches[0])
            for st in side:
                main.wait_stream(st)
        else:
            for parts in batches:
                _native_muon_bucket(optimizer, group, parts)
        return
    world, rank = dist.get_world_size(), dist.get_rank()
    owners = muon_owners(group, path, world)
    owned = {key: [params[i] for i in idx if owners[i] == rank] for key, idx in buckets.items()}
    if path == "slab":
        assert slab is not None
        for parts in _batches(owned):
            _native_muon_bucket(optimizer, group, parts, slab=slab)
        for i, p in enumerate(params):
            if owners[i] != rank and getattr(p, "_kb_shadow", None) is not None:
                p._kb_shadow_version = -1  # rewritten by its owner: recast before the next forward
        return
    for parts in _batches(owned):
        _native_muon_bucket(optimizer, group, parts)
    for (R, C), idx in buckets.items():
        mine = owned[(R, C)]
        per_rank = (len(idx) + world - 1) // world
        send = torch.zeros((per_rank, R * C), device=params[0].device, dtype=torch.float32)
        for j, p in enumerate(mine):
            send[j].copy_(p.detach().reshape(-1))
        recv = torch.empty((world * per_rank, R * C), device=send.device, dtype=torch.float32)
        dist.all_gather_into_tensor(recv, send)
        for k, i in enumerate(idx):
            if k % world == rank:
                continue
            params[i].detach().view(-1).copy_(recv[(k % world) * per_rank + k // world])


def _sharded_adam_group(optimizer, group, slab) -> None:
    """AdamW on this rank's shard of every tensor of an Adam group, published into every rank's copy.

    The gradient sync reduce-scattered these tensors (``shard_bounds`` per
    tensor), so only the shard of ``p.grad`` holds averaged values here.
    """

    from ..ops._ext import native
    from ..parallel.symm import shard_bounds

    params = list(group["params"])
    if not params:
        return
    world, rank = dist.get_world_size(), dist.get_rank()
    grads, m, v, steps, lo, hi = [], [], [], [], [], []
    for p in params:
        _ensure_grad(p)
        st = optimizer.state[p]
        if "exp_avg" not in st:
            st["exp_avg"] = torch.zeros_like(p)
            st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] = 0
        st["step"] = int(st["step"]) + 1
        a, b = shard_bounds(p.numel(), world, rank)
        grads.append(p.grad)
        m.append(st["exp_avg"])
        v.append(st["exp_avg_sq"])
        steps.append(int(st["step"]))
        lo.append(a)
        hi.append(b)
    b1, b2 = group["betas"]
    ws = slab.ws
    native().adam_shard_gather(params, grads, m, v, lo, hi, steps, _clip_scale(optimizer),
                               getattr(optimizer, "kb_skip_flag", None), float(group["lr"]), float(b1), float(b2),
                               float(group["eps"]), float(group["weight_decay"]), ws.bases, ws.mc_base, ws.rank,
                               ws.nbytes)
    for p in params:
        if getattr(p, "_kb_shadow", None) is not None:
            p._kb_shadow_version = -1  # only this rank's shard was written locally: recast before the next forward


def _optimizer_slab(optimizer, params: List[torch.nn.Parameter]):
    """The optimizer's symmetric parameter slab holding ``params`` (built, or rebuilt, on demand)."""

    slab = optimizer.__dict__.get("_kb_slab")
    if slab is None or not slab.holds(params):
        from ..parallel.symm import SymmetricParamSlab

        slab = SymmetricParamSlab(params, params[0].device)
        optimizer.__dict__["_kb_slab"] = slab
    return slab


def _run_groups(optimizer, muon_fn: Callable, normuon: bool, distributed: bool,
                skip: Optional[torch.Tensor] = None) -> None:
    plan = getattr(optimizer, "_kb_plan", None) if distributed else None
    shard_adam = bool(plan and plan["shard_rest"])
    paths = []
    slab_params: List[torch.nn.Parameter] = []
    for group in optimizer.param_groups:
        if group.get("use_muon", True):
            path = _muon_path(group, normuon, distributed)
            if path == "slab":
                slab_params += list(group["params"])
        else:
            native_ok = _native_ready(group["params"]) and not _foreach_adam_enabled(group)
            path = ("sharded" if shard_adam else "native") if native_ok else "ref"
            if path == "sharded":
                slab_params += list(group["params"])
        paths.append(path)
    if shard_adam and "ref" in [p for g, p in zip(optimizer.param_groups, paths) if not g.get("use_muon", True)]:
        raise RuntimeError("the gradient sync reduce-scattered the Adam tensors, but an Adam group cannot take "
                           "the sharded native path")
    if skip is not None and "ref" in paths:
        # The PyTorch paths cannot skip on the device: read the flag on the host.
        if float(skip.sum()) != 0.0:
            return
        skip = None
    slab = _optimizer_slab(optimizer, slab_params) if slab_params else None
    from ..ops._ext import native

    C = native() if skip is not None else None
    if C is not None:
        C.set_step_skip(skip)
    try:
        _run_paths(optimizer, muon_fn, distributed, paths, slab)
    finally:
        if C is not None:
            C.set_step_skip(None)
    if slab is not None:
        slab.barrier()  # every rank's peer stores of this step have landed


def _run_paths(optimizer, muon_fn: Callable, distributed: bool, paths: List[str], slab) -> None:
    ran = getattr(optimizer, "_kb_adam_ran", None)
    for group, path in zip(optimizer.param_groups, paths):
        params = group["params"]
        if group.get("use_muon", True):
            with _profile_range("optimizer.muon.update"):
                if path == "ref":
                    _ref_muon_group(optimizer, group, muon_fn, distributed)
                else:
                    _native_muon_group(optimizer, group, path, slab)
        else:
            with _profile_range("optimizer.adam.update"):
                if path == "sharded":
                    _sharded_adam_group(optimizer, group, slab)
                elif path == "native":
                    _native_adam_group(optimizer, group)
                else:
                    _ref_adam_group(optimizer, group)
            if ran is not None and path != "ref":
                ran.append(group)


def gradient_plan(optimizer, world: int) -> Tuple[Dict[int, int], bool]:
    """Where the data-parallel sync must deliver each reduced gradient for this optimizer.

    Returns (owners, shard_rest): ``owners`` maps ``id(param)`` of every
    distributed Muon matrix to the rank whose step reads its gradient, and
    ``shard_rest`` says whether every Adam tensor can be reduce-scattered
    (its update runs sharded, ``_sharded_adam_group``). Both are empty/False
    when a group needs gradients everywhere (non-native or foreach Adam
    groups, a non-distributed optimizer).
    """

    if not (getattr(optimizer, "_distributed", False) and world > 1):
        return {}, False
    normuon = bool(getattr(optimizer, "_normuon", False))
    owners: Dict[int, int] = {}
    shard_rest = True
    for group in optimizer.param_groups:
        params = list(group["params"])
        if group.get("use_muon", True):
            path = _muon_path(group, normuon, True)
            for p, r in zip(params, muon_owners(group, path, world)):
                owners[id(p)] = r
        elif not (_native_ready(params) and not _foreach_adam_enabled(group) and _slab_ok(params)):
            shard_rest = False
    if not shard_rest:
        # Replicated Adam steps read every gradient; Muon owners still only need their own matrices.
        pass
    return owners, shard_rest


def _sorted_desc(params: Iterable[torch.nn.Parameter]) -> List[torch.nn.Parameter]:
    return sorted(list(params), key=lambda x: x.size(), reverse=True)


def _muon_defaults(group: Dict[str, Any], with_beta2: bool = False) -> None:
    group.setdefault("lr", 0.02)
    group.setdefault("momentum", 0.95)
    group.setdefault("weight_decay", 0)
    if with_beta2:
        group.setdefault("beta2", 0.95)


def _adam_defaults(group: Dict[str, Any]) -> None:
    group.setdefault("lr", 3e-4)
    group.setdefault("betas", (0.9, 0.95))
    group.setdefault("eps", 1e-10)
    group.setdefault("weight_decay", 0)


def _closure(closure):
    if closure is None:
        return None
    with torch.enable_grad():
        return closure()


class _KbOptimizer(torch.optim.Optimizer):
    """Base: fused-path hooks consumed by one step, device-side skip, and sharded-state handling.

    Hooks set before ``step`` and cleared by it: ``kb_grad_scale`` (clip
    coefficient, a device scalar applied when each gradient is read),
    ``kb_ema`` (a GPU EMA update fused into the update kernels) and
    ``kb_skip`` (a device flag; non-zero makes every kernel of the step
    return before touching any state). ``GradScaler.step`` hands over its
    found-inf flag the same way (``_step_supports_amp_scaling``: it sets
    ``found_inf`` / ``grad_scale`` instead of reading found-inf on the host),
    so a skipped step costs no host synchronisation. A step skipped on the
    device still advanced the host-side Adam step counters;
    ``kb_rollback_step`` undoes that once the caller has read the flag.
    """

    kb_fused = True
    _normuon = False
    _distributed = False
    _step_supports_amp_scaling = True

    def _distributed_now(self) -> bool:
        return self._distributed and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1

    def _skip_flag(self) -> Optional[torch.Tensor]:
        flags = [f for f in (getattr(self, "kb_skip", None), getattr(self, "found_inf", None)) if f is not None]
        if not flags:
            return None
        flag = flags[0].float().reshape(-1)[:1]
        for f in flags[1:]:
            flag = flag + f.float().reshape(-1)[:1]
        return flag.contiguous()

    @torch.no_grad()
    def step(self, closure=None):
        loss = _closure(closure)
        fn = _normuon_param_update if self._normuon else _muon_param_update
        skip = self._skip_flag()
        grad_scale = getattr(self, "grad_scale", None)  # GradScaler: gradients not unscaled yet
        if grad_scale is not None:
            inv = grad_scale.double().reciprocal().float().reshape(1)
            coef = getattr(self, "kb_grad_scale", None)
            self.kb_grad_scale = inv if coef is None else coef * inv
        self._kb_adam_ran: List[Dict[str, Any]] = []
        try:
            _run_groups(self, fn, self._normuon, self._distributed_now(), skip)
        finally:
            self.kb_grad_scale = None
            self.kb_ema = None
            self.kb_skip = None
        return loss

    def kb_rollback_step(self) -> None:
        """Undo the host-side step counters of the last step, which its kernels skipped on the device."""

        for group in getattr(self, "_kb_adam_ran", []):
            for p in group["params"]:
                st = self.state.get(p)
                if st and "step" in st:
                    st["step"] = int(st["step"]) - 1
        self._kb_adam_ran = []

    def kb_commit_gradient_plan(self, world: int) -> Tuple[Dict[int, int], bool]:
        """Fix where reduced gradients must arrive (see ``gradient_plan``); later steps rely on it."""

        owners, shard_rest = gradient_plan(self, world)
        self._kb_plan = {"world": world, "owners": dict(owners), "shard_rest": bool(shard_rest)}
        return owners, shard_rest

    def _muon_state_keys(self) -> List[str]:
        return ["momentum_buffer", "second_momentum_buffer"] if self._normuon else ["momentum_buffer"]

    @torch.no_grad()
    def gathered_state_dict(self) -> Dict[str, Any]:
        """The full optimizer state, on every rank (a collective: every rank must call it).

        A distributed step keeps each Muon matrix's momentum only on its
        owner, and with a sharded Adam step each rank's Adam moments are
        current only on its shard. This gathers both (owners' buffers summed
        with zeros elsewhere, which is exact) so the returned state dict has
        the layout and values of a single-process run: every Muon matrix's
        ``momentum_buffer`` in the reference's parameter order, full
        ``exp_avg`` / ``exp_avg_sq``. Non-distributed: ``state_dict()``.
        """

        if not self._distributed_now():
            return self.state_dict()
        world, rank = dist.get_world_size(), dist.get_rank()
        plan = getattr(self, "_kb_plan", None) or {}
        temp: List[torch.nn.Parameter] = []
        for group in self.param_groups:
            params = list(group["params"])
            if not params:
                continue
            dev = params[0].device
            if group.get("use_muon", True):
                owners = muon_owners(group, _muon_path(group, self._normuon, True), world)
                for key in self._muon_state_keys():
                    present = torch.tensor([float(owners[i] == rank and key in self.state.get(p, {}))
                                            for i, p in enumerate(params)], device=dev)
                    dist.all_reduce(present)
                    for i, p in enumerate(params):
                        if float(present[i]) == 0.0:
                            continue
                        st = self.state[p]
                        mine = owners[i] == rank
                        if key == "momentum_buffer":
                            shape = p.shape
                        else:
                            shape = (p.shape[0], 1) if p.ndim > 2 else (*p.shape[:-1], 1)
                        buf = st[key].detach().clone() if mine else torch.zeros(shape, device=dev, dtype=p.dtype)
                        dist.all_reduce(buf)
                        if not mine:
                            st[key] = buf
                            temp.append(p)
            elif plan.get("shard_rest"):
                from ..parallel.symm import shard_bounds

                for p in params:
                    st = self.state.get(p)
                    if not st or "exp_avg" not in st:
                        continue
                    lo, hi = shard_bounds(p.numel(), world, rank)
                    for key in ("exp_avg", "exp_avg_sq"):
                        flat = st[key].view(-1)
                        flat[:lo].zero_()
                        flat[hi:].zero_()
                        dist.all_reduce(st[key])  # every rank now holds the complete moments
        sd = self.state_dict()
        for p in temp:  # borrowed from the owners for this dict only
            for key in self._muon_state_keys():
                self.state[p].pop(key, None)
            if not self.state[p]:
                del self.state[p]
        return sd

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None:
        super().load_state_dict(state_dict)
        if not self._distributed_now():
            return
        # A gathered checkpoint holds every matrix's momentum: keep only the owned ones.
        world, rank = dist.get_world_size(), dist.get_rank()
        for group in self.param_groups:
            if not group.get("use_muon", True):
                continue
            owners = muon_owners(group, _muon_path(group, self._normuon, True), world)
            for p, r in zip(group["params"], owners):
                if r != rank and p in self.state:
                    del self.state[p]


class Muon(_KbOptimizer):
    """Distributed Muon for hidden matrices (``lr`` in spectral-norm units)."""

    _distributed = True

    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95):
        params = list(params)
        assert len(params) >= 1 and isinstance(params[0], torch.nn.Parameter)
        super().__init__(_sorted_desc(params), dict(lr=lr, weight_decay=weight_decay, momentum=momentum))


class SingleDeviceMuon(_KbOptimizer):
    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95):
        super().__init__(params, dict(lr=lr, weight_decay=weight_decay, momentum=momentum))


class NorMuon(_KbOptimizer):
    _distributed = True
    _normuon = True

    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95, beta2=0.95):
        params = list(params)
        assert len(params) >= 1 and isinstance(params[0], torch.nn.Parameter)
        super().__init__(_sorted_desc(params), dict(lr=lr, weight_decay=weight_decay, momentum=momentum, beta2=beta2))


class SingleDeviceNorMuon(_KbOptimizer):
    _normuon = True

    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95, beta2=0.95):
        super().__init__(params, dict(lr=lr, weight_decay=weight_decay, momentum=momentum, beta2=beta2))


def _init_groups(groups: Sequence[Dict[str, Any]], *, with_beta2: bool, sort_muon: bool) -> None:
    for g in groups:
        assert "use_muon" in g
        if g["use_muon"]:
            if sort_muon:
                g["params"] = _sorted_desc(g["params"])
            _muon_defaults(g, with_beta2)
        else:
            _adam_defaults(g)


class MuonWithAuxAdam(_KbOptimizer):
    """Muon on ``use_muon`` groups and Adam on the rest (distributed Muon sharding)."""

    _distributed = True

    def __init__(self, param_groups):
        _init_groups(param_groups, with_beta2=False, sort_muon=True)
        super().__init__(param_groups, dict())


class SingleDeviceMuonWithAuxAdam(_KbOptimizer):
    def __init__(self, param_groups):
        _init_groups(param_groups, with_beta2=False, sort_muon=False)
        super().__init__(param_groups, dict())


class NorMuonWithAuxAdam(_KbOptimizer):
    _distributed = True
    _normuon = True

    def __init__(self, param_groups):
        _init_groups(param_groups, with_beta2=True, sort_muon=True)
        super().__init__(param_groups, dict())


class SingleDeviceNorMuonWithAuxAdam(_KbOptimizer):
    _normuon = True

    def __init__(self, param_groups):
        _init_groups(param_groups, with_beta2=True, sort_muon=False)
        super().__init__(param_groups, dict())


class FusedAdamW(_KbOptimizer):
    """AdamW (decoupled weight decay, bias-corrected moments) on the native multi-tensor kernel.

    The update is ``torch.optim.AdamW``'s (reference koochak/optim/build.py:174-177
    builds that class): ``p *= 1 - lr * wd``, then ``p -= lr * m_hat /
    (sqrt(v_hat) + eps)``. All tensors of a group are updated by one launch,
    which also applies a clip coefficient handed over as a device scalar and
    the fused EMA. Under data parallelism the gradient sync may reduce-scatter
    the gradients and the step then updates this rank's shard and publishes
    it to the peers (the sharded Adam path). The state dict has
    ``torch.optim.AdamW``'s keys (``step``, ``exp_avg``, ``exp_avg_sq``).
    """

    _distributed = True

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 1e-2):
        params = list(params)
        groups = params if params and isinstance(params[0], dict) else [{"params": params}]
        for g in groups:
            g["use_muon"] = False
        super().__init__(groups, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))

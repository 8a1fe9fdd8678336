"""The KB_DEBUG_BOUNDS build: odd shapes pass clean, and a short declared extent is caught, not accessed.

The debug variant of the native library (``csrc/_build_debug``, loaded when
``KOOCHAK_DEBUG_BOUNDS=1``) checks every GEMM epilogue tile and every
sharded-Adam work item against the extent the host declared for its buffers.
Each case runs in a child process that loads only that variant:

* GEMMs at odd sizes (not multiples of 64 or 128; transposed operands;
  fp32 stream-K outputs with D; batched) match the fp32 PyTorch product and
  leave the status word clear;
* with the declared extents shortened by one element (the buffers keep their
  real size, so nothing outside an allocation is touched either way) the
  GEMM records status 7 at the output site with the last row's index, and
  the sharded-Adam step records it at its own site.
"""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = textwrap.dedent(
    """
    import torch
    from koochak_b200.ops import functional as kf
    from koochak_b200.ops._ext import native

    C = native()
    assert C.debug_bounds_enabled(), "the debug-bounds variant was not loaded"
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)

    def status():
        torch.cuda.synchronize()
        return C.read_and_clear_status(0), C.read_debug_bounds_detail(0)

    # 1. odd shapes, clean status, correct results
    # (M-major and N-major operands need 16-byte rows: M or N a multiple of 8 there)
    cases = [(200, 136, 72, False, False, torch.bfloat16), (136, 264, 200, True, False, torch.bfloat16),
             (77, 96, 520, False, True, torch.float32), (304, 40, 136, True, True, torch.float32)]
    for M, N, K, amn, bmn, odt in cases:
        a = torch.randn((K, M) if amn else (M, K), device=dev).bfloat16()
        b = torch.randn((K, N) if bmn else (N, K), device=dev).bfloat16()
        d = torch.randn(M, N, device=dev, dtype=odt)
        out = kf.gemm(a, b, a_mn_major=amn, b_mn_major=bmn, d=d, beta=0.5, out_dtype=odt)
        ref = kf.gemm_ref(a, b, a_mn_major=amn, b_mn_major=bmn, d=d, beta=0.5)
        code, detail = status()
        assert code == 0, (M, N, K, code, detail)
        err = float((out.float() - ref).abs().max() / ref.abs().max())
        assert err < 2e-2, (M, N, K, err)
    a = torch.randn(3, 130, 72, device=dev).bfloat16()
    b = torch.randn(3, 136, 72, device=dev).bfloat16()
    out = kf.gemm(a, b)
    code, _ = status()
    assert code == 0
    assert float((out.float() - kf.gemm_ref(a, b)).abs().max()) < 0.5

    # 2. declared extents one element short: the GEMM epilogue check fires
    M, N, K = 130, 128, 64
    a = torch.randn(M, K, device=dev).bfloat16()
    b = torch.randn(N, K, device=dev).bfloat16()
    out = torch.zeros(M, N, device=dev, dtype=torch.bfloat16)
    C.set_debug_extent_slack(1)
    try:
        kf.gemm(a, b, out=out)
        code, (site, index, extent) = status()
    finally:
        C.set_debug_extent_slack(0)
    assert code == 7, code
    assert site == 1, site  # GEMM output
    assert extent == M * N - 1 and index >= extent, (index, extent)
    # the rows of the tiles that passed the check were written
    assert float((out[:96].float() - kf.gemm_ref(a[:96], b)).abs().max()) < 0.5

    # 3. the sharded-Adam step (one rank: the slab is local) checks its work items
    slab = torch.zeros(4096 + 1000, device=dev)
    p = slab[:4096].view(64, 64)
    g = torch.randn(64, 64, device=dev)
    m = torch.zeros_like(g)
    v = torch.zeros_like(g)
    base = slab.data_ptr()
    C.set_debug_extent_slack(1)
    try:
        C.adam_shard_gather([p], [g], [m], [v], [0], [4096], [1], None, None, 1e-3, 0.9, 0.95, 1e-8, 0.0,
                            [base], 0, 0, slab.numel() * 4)
        code, (site, index, extent) = status()
    finally:
        C.set_debug_extent_slack(0)
    assert code == 7 and site == 6, (code, site)
    C.adam_shard_gather([p], [g], [m], [v], [0], [4096], [1], None, None, 1e-3, 0.9, 0.95, 1e-8, 0.0,
                        [base], 0, 0, slab.numel() * 4)
    code, _ = status()
    assert code == 0
    assert float(p.abs().max()) > 0
    print("debug-bounds ok")
    """
)


def test_debug_bounds_variant():
    env = dict(os.environ, KOOCHAK_DEBUG_BOUNDS="1", PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    proc = subprocess.run([sys.executable, "-c", _CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=600)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "debug-bounds ok" in proc.stdout

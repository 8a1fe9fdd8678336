"""Native sm_100a kernels against plain-PyTorch fp32 references of the same ops."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _kf():
    from koochak_b200.ops import functional as kf

    return kf


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


@pytest.fixture(autouse=True)
def _status_clean():
    from koochak_b200.ops import check_status

    yield
    torch.cuda.synchronize()
    check_status()


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (300, 200, 136), (1000, 776, 520), (2048, 2304, 768)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("block_n", [128, 256])
def test_gemm_layouts(M, N, K, a_mn, b_mn, block_n):
    kf = _kf()
    torch.manual_seed(0)
    if (a_mn and M % 8) or (b_mn and N % 8):
        pytest.skip("MN-major operands need 16-byte aligned rows")
    a = (torch.randn(K, M) if a_mn else torch.randn(M, K)).to(DEV, torch.bfloat16)
    b = (torch.randn(K, N) if b_mn else torch.randn(N, K)).to(DEV, torch.bfloat16)
    out = kf.gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn, out_dtype=torch.float32, block_n=block_n)
    ref = kf.gemm_ref(a, b, a_mn_major=a_mn, b_mn_major=b_mn)
    assert _rel(out, ref) < 1e-4


def test_gemm_epilogues_and_batch():
    kf = _kf()
    torch.manual_seed(1)
    M, N, K = 512, 384, 256
    a = torch.randn(M, K, device=DEV).bfloat16()
    b = torch.randn(N, K, device=DEV).bfloat16()
    bias = torch.randn(N, device=DEV)
    d = torch.randn(M, N, device=DEV).bfloat16()
    out = kf.gemm(a, b, d=d, alpha=0.5, beta=2.0, bias=bias)
    assert _rel(out, kf.gemm_ref(a, b, d=d, alpha=0.5, beta=2.0, bias=bias)) < 1e-2
    aux = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    g = kf.gemm(a, b, bias=bias, aux=aux, act=kf.ACT_GELU)
    ref_g, ref_pre = kf.gemm_ref(a, b, bias=bias, act=kf.ACT_GELU)
    assert _rel(g, ref_g) < 1e-2 and _rel(aux, ref_pre) < 1e-2
    h = torch.randn(M, N, device=DEV).bfloat16()
    gb = kf.gemm(a, b, d=h, act=kf.ACT_GELU_BWD)
    assert _rel(gb, kf.gemm_ref(a, b, d=h, act=kf.ACT_GELU_BWD)) < 1e-2
    ab = torch.randn(3, 256, 320, device=DEV).bfloat16()
    bb = torch.randn(3, 192, 320, device=DEV).bfloat16()
    ob = kf.gemm(ab, bb, out_dtype=torch.float32)
    assert _rel(ob, torch.bmm(ab.float(), bb.float().transpose(1, 2))) < 1e-4
    # fp32 accumulate into an existing output (D = C)
    c = torch.randn(M, N, device=DEV)
    ref = c + kf.gemm_ref(a, b)
    kf.gemm(a, b, out=c, d=c, beta=1.0)
    assert _rel(c, ref) < 1e-4


@pytest.mark.parametrize("C", [64, 768, 1000, 1280, 2048, 3072, 4096])
@pytest.mark.parametrize("rms", [False, True])
def test_norm_forward_backward(C, rms):
    kf = _kf()
    torch.manual_seed(2)
    M = 333
    x = torch.randn(M, C, device=DEV)
    w = torch.randn(C, device=DEV)
    b = None if rms else torch.randn(C, device=DEV)
    y, mean, rstd = kf.norm_forward(x, w, b, 1e-5, rms=rms, out_dtype=torch.bfloat16)
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    br = None if rms else b.clone().requires_grad_(True)
    yr = kf.rms_norm_ref(xr, wr, 1e-5) if rms else kf.layer_norm_ref(xr, wr, br, 1e-5)
    assert _rel(y, yr) < 1e-2
    dy = torch.randn(M, C, device=DEV).bfloat16()
    dres = torch.randn(M, C, device=DEV)
    dx, dw, db = kf.norm_backward(dy, x, w, mean, rstd, rms=rms, dres=dres, dx_dtype=torch.float32)
    yr.backward(dy.float())
    assert _rel(dx, xr.grad + dres) < 1e-3
    assert _rel(dw, wr.grad) < 1e-3
    if not rms:
        assert _rel(db, br.grad) < 1e-3


@pytest.fixture(params=["tcgen05", "mma_sync"])
def attn_impl(request):
    from koochak_b200.ops import native

    native().attention_set_impl(0 if request.param == "tcgen05" else 1)
    yield request.param
    native().attention_set_impl(0)


@pytest.mark.parametrize("B,S,H,D,causal", [(2, 256, 4, 64, True), (2, 200, 3, 64, False), (1, 384, 2, 128, True),
                                            (3, 197, 2, 64, False), (1, 130, 2, 128, False),
                                            (1, 1100, 2, 64, True), (1, 700, 1, 128, False)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_flash_attention(B, S, H, D, causal, dtype, attn_impl):
    kf = _kf()
    torch.manual_seed(3)
    qkv = torch.randn(B, S, 3, H, D, device=DEV).to(dtype)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    o, lse = kf.flash_attention_forward(q, k, v, causal=causal)
    qr, kr, vr = (t.float().detach().requires_grad_(True) for t in (q, k, v))
    ref = kf.attention_ref(qr, kr, vr, causal=causal)
    assert _rel(o, ref) < 2e-2
    sc = torch.einsum("bqhd,bkhd->bhqk", qr, kr) / math.sqrt(D)
    if causal:
        sc = sc.masked_fill(torch.ones(S, S, device=DEV, dtype=torch.bool).triu(1), float("-inf"))
    assert (lse - torch.logsumexp(sc, -1)).abs().max().item() < 2e-2
    do = torch.randn_like(o)
    ref.backward(do.float())
    dqkv = torch.empty_like(qkv)
    kf.flash_attention_backward(q, k, v, o, do, lse, causal=causal, dq=dqkv[:, :, 0], dk=dqkv[:, :, 1],
                                dv=dqkv[:, :, 2])
    assert _rel(dqkv[:, :, 0], qr.grad) < 3e-2
    assert _rel(dqkv[:, :, 1], kr.grad) < 3e-2
    assert _rel(dqkv[:, :, 2], vr.grad) < 3e-2


def test_cross_entropy_and_embedding():
    kf = _kf()
    torch.manual_seed(4)
    M, V = 300, 1000
    vpad = 1024
    logits = torch.randn(M, vpad, device=DEV).bfloat16()
    tgt = torch.randint(0, V, (M,), device=DEV)
    tgt[5] = -100
    loss, lse = kf.cross_entropy_forward(logits, tgt, V)
    lref = logits[:, :V].float().requires_grad_(True)
    ref = F.cross_entropy(lref, tgt, reduction="none")
    assert (loss - ref).abs().max().item() < 1e-3
    n = (tgt != -100).sum().float()
    ref.sum().div(n).backward()
    g = (1.0 / n).reshape(1).to(DEV)
    kf.cross_entropy_backward_(logits, tgt, lse, g, V)
    assert (logits[:, :V].float() - lref.grad).abs().max().item() < 1e-3
    wte = torch.randn(50, 64, device=DEV)
    wpe = torch.randn(16, 64, device=DEV)
    idx = torch.randint(0, 50, (3, 16), device=DEV)
    out = kf.embedding_forward(idx, wte, wpe, 16)
    assert torch.allclose(out, wte[idx] + wpe[None], atol=1e-6)
    dout = torch.randn(3, 16, 64, device=DEV)
    dwte, dwpe = kf.embedding_backward(idx, dout, 50, 16, 16)
    ref_wte = torch.zeros_like(wte).index_add_(0, idx.reshape(-1), dout.reshape(-1, 64))
    assert torch.allclose(dwte, ref_wte, atol=1e-4)
    assert torch.allclose(dwpe, dout.sum(0), atol=1e-4)
    gbias = torch.randn(777, 300, device=DEV).bfloat16()
    assert _rel(kf.bias_grad(gbias), gbias.float().sum(0)) < 1e-4


@pytest.mark.parametrize("F", [96, 100, 5504])
@pytest.mark.parametrize("M", [37, 5001])
def test_swiglu(F, M):
    """Vectorised (F % 8 == 0) and scalar (F = 100) SwiGLU against the fp32 formula; with 5001 rows the
    vectorised kernels take two rows per step and an odd tail."""

    kf = _kf()
    torch.manual_seed(5)
    gu = torch.randn(M, 2 * F, device=DEV).bfloat16()
    assert _rel(kf.swiglu_forward(gu), kf.swiglu_ref(gu)) < 1e-2
    gr = gu.float().requires_grad_(True)
    dh = torch.randn(M, F, device=DEV).bfloat16()
    kf.swiglu_ref(gr).backward(dh.float())
    assert _rel(kf.swiglu_backward(gu, dh), gr.grad) < 2e-2


@pytest.mark.parametrize("D", [64, 128, 24])
def test_rope(D):
    """RoPE in place, forward and inverse; D = 24 takes the scalar kernel. The q and k heads of a fused
    [B, S, 3, H, D] projection are rotated by one call on their [B, S, 2H, D] view, as the Llama layer does."""

    kf = _kf()
    torch.manual_seed(5)
    B, S, H = 2, 32, 3
    qkv = torch.randn(B, S, 3, H, D, device=DEV).bfloat16()
    pos = torch.arange(S, device=DEV).float()[:, None]
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=DEV).float() / D))
    cos, sin = torch.cos(pos * inv).contiguous(), torch.sin(pos * inv).contiguous()
    ref_q, ref_k = kf.rope_ref(qkv[:, :, 0], cos, sin), kf.rope_ref(qkv[:, :, 1], cos, sin)
    y = qkv.clone()
    kf.rope_apply_(y[:, :, :2].view(B, S, 2 * H, D), cos, sin)
    assert _rel(y[:, :, 0], ref_q) < 1e-2 and _rel(y[:, :, 1], ref_k) < 1e-2
    assert torch.equal(y[:, :, 2], qkv[:, :, 2])
    kf.rope_apply_(y[:, :, :2].view(B, S, 2 * H, D), cos, sin, inverse=True)
    assert _rel(y, qkv) < 2e-2


def test_optimizer_kernels_match_reference():
    from koochak_b200.optim.muon import SingleDeviceMuonWithAuxAdam

    torch.manual_seed(6)
    shapes = [(96, 64), (64, 160), (64, 160), (32,), (128, 48, 2), (64, 96)]

    def make():
        torch.manual_seed(7)
        return [torch.nn.Parameter(torch.randn(*s) * 0.1) for s in shapes]

    grads = [torch.randn(*s) * 1e-2 for s in shapes]

    def groups(ps):
        muon = [p for p in ps if p.ndim >= 2]
        adam = [p for p in ps if p.ndim < 2]
        return [dict(params=adam, lr=1e-3, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01, use_muon=False),
                dict(params=muon, lr=0.02, momentum=0.95, weight_decay=0.01, use_muon=True)]

    cpu = make()
    gpu = [torch.nn.Parameter(p.detach().to(DEV)) for p in make()]
    o_cpu = SingleDeviceMuonWithAuxAdam(groups(cpu))
    o_gpu = SingleDeviceMuonWithAuxAdam(groups(gpu))
    for _ in range(3):
        for p, g in zip(cpu, grads):
            p.grad = g.clone()
        for p, g in zip(gpu, grads):
            p.grad = g.to(DEV).clone()
        o_cpu.step()
        o_gpu.step()
    for pc, pg in zip(cpu, gpu):
        assert _rel(pg.detach().cpu(), pc.detach()) < 2e-2
    sd = o_gpu.state_dict()
    assert all("momentum_buffer" in s or "exp_avg" in s for s in sd["state"].values())


def test_grad_gate_and_ema_kernels():
    from koochak_b200.optim.grad_clip import clip_grad_norm_, fused_grad_gate
    from koochak_b200.ops import native

    torch.manual_seed(8)
    grads = [torch.randn(n, device=DEV) for n in (10, 1000, 70000)]
    ref_grads = [g.clone() for g in grads]
    params = [torch.nn.Parameter(torch.zeros_like(g)) for g in ref_grads]
    for p, g in zip(params, ref_grads):
        p.grad = g
    ref = clip_grad_norm_(params, 1.0)
    res = fused_grad_gate(grads, max_norm=1.0, check_finite=True)
    assert abs(res.stats.norm - ref.norm) / ref.norm < 1e-5
    assert abs(res.stats.coefficient - ref.coefficient) / ref.coefficient < 1e-5
    grads[1][3] = float("inf")
    with pytest.raises(FloatingPointError):
        fused_grad_gate(grads, max_norm=1.0, check_finite=True)
    sh = [torch.randn(100, device=DEV), torch.randn(7, 9, device=DEV)]
    ps = [torch.randn(100, device=DEV), torch.randn(7, 9, device=DEV)]
    exp = [0.9 * s + 0.1 * p for s, p in zip(sh, ps)]
    native().ema_update(sh, ps, 0.9)
    for a, b in zip(sh, exp):
        assert torch.allclose(a, b, atol=1e-6)


def test_gpt2_native_matches_reference_path():
    from koochak_b200.models import GPT2

    torch.manual_seed(9)
    model = GPT2(n_layer=2, n_head=4, n_embd=256, vocab_size=1000, block_size=128).to(DEV)
    idx = torch.randint(0, 1000, (2, 128), device=DEV)
    tgt = torch.randint(0, 1000, (2, 128), device=DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = model(idx, tgt)
    loss.backward()
    g_native = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    ref = model._forward_reference(idx, tgt, -100)  # fp32 reference math
    ref.backward()
    assert abs(loss.item() - ref.item()) < 2e-2
    for n, p in model.named_parameters():
        assert _rel(g_native[n], p.grad) < 0.08, n


@pytest.mark.parametrize("M,N,K", [(2304, 768, 16384), (768, 3072, 4096), (520, 776, 2000)])
@pytest.mark.parametrize("block_n", [0, 128, -256])
def test_gemm_stream_k_fp32(M, N, K, block_n):
    """fp32 outputs spread over all SMs by K-iterations (stream-K), with bias and beta * D."""
    kf = _kf()
    torch.manual_seed(12)
    a = torch.randn(K, M, device=DEV).bfloat16()
    b = torch.randn(K, N, device=DEV).bfloat16()
    ref = kf.gemm_ref(a, b, a_mn_major=True, b_mn_major=True)
    out = kf.gemm(a, b, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32, block_n=block_n)
    assert _rel(out, ref) < 1e-4
    d = torch.randn(M, N, device=DEV)
    bias = torch.randn(N, device=DEV)
    out2 = kf.gemm(a, b, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32, d=d, beta=0.5, bias=bias,
                   block_n=block_n)
    assert _rel(out2, ref + bias + 0.5 * d) < 1e-4
    acc = d.clone()
    kf.gemm(a, b, a_mn_major=True, b_mn_major=True, out=acc, d=acc, beta=1.0, block_n=block_n)
    assert _rel(acc, ref + d) < 1e-4


def test_patchify_matches_reference():
    kf = _kf()
    img = torch.randn(3, 3, 64, 48, device=DEV)
    for dt in (torch.float16, torch.bfloat16):
        got = kf.patchify(img, 16, dt)
        assert torch.equal(got, kf.patchify_ref(img, 16).to(dt))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_vit_native_matches_reference_path(dtype):
    from koochak_b200.models import ViT

    torch.manual_seed(6)
    model = ViT(depth=2, image_size=64, num_classes=100, dim=256, n_head=4).to(DEV)
    x = torch.randn(4, 3, 64, 64, device=DEV)
    y = torch.randint(0, 100, (4,), device=DEV)
    with torch.autocast("cuda", dtype=dtype):
        loss = model(x, y)
    loss.backward()
    g_native = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    ref = model._forward_reference(x, y)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 3e-2
    for n, p in model.named_parameters():
        assert _rel(g_native[n], p.grad) < 0.08, n


@pytest.mark.parametrize("head_dim", [64, 128])
def test_llama_native_matches_reference_path(head_dim):
    from koochak_b200.models import Llama

    torch.manual_seed(5)
    model = Llama(n_layer=2, n_head=256 // head_dim, dim=256, ffn_dim=688, vocab_size=1024, max_seq_len=128).to(DEV)
    idx = torch.randint(0, 1024, (2, 128), device=DEV)
    tgt = torch.randint(0, 1024, (2, 128), device=DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = model(idx, tgt)
    loss.backward()
    g_native = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    cos, sin = model.rope(128, DEV)
    ref = model._forward_reference(idx, tgt, -100, cos, sin)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 2e-2
    for n, p in model.named_parameters():
        assert _rel(g_native[n], p.grad) < 0.08, n


def test_llama_gradient_accumulation_in_place_matches_autograd():
    """Later micro-steps add weight gradients straight into .grad (GEMM with the old gradient as D);
    the result matches autograd's accumulation, which a hook on every parameter forces in the twin."""

    from koochak_b200.models import Llama

    def make():
        torch.manual_seed(6)
        return Llama(n_layer=2, n_head=4, dim=256, ffn_dim=688, vocab_size=1024, max_seq_len=128).to(DEV)

    ours, twin = make(), make()
    for p in twin.parameters():
        p.register_post_accumulate_grad_hook(lambda _p: None)
    g = torch.Generator(device="cpu").manual_seed(3)
    batches = [torch.randint(0, 1024, (2, 129), generator=g).to(DEV) for _ in range(3)]
    first_ptr = None
    for i, b in enumerate(batches):
        for m in (ours, twin):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = m(b[:, :-1], b[:, 1:]) / 3
            loss.backward()
        wq = ours.model.layers[0].self_attn.q_proj.weight
        if i == 0:
            first_ptr = wq.grad.data_ptr()
        else:
            assert wq.grad.data_ptr() == first_ptr  # accumulated in place, not replaced
    # bf16 forward/backward with fp32 atomics is not bitwise reproducible between two models: compare norms
    for (n, p), q in zip(ours.named_parameters(), twin.parameters()):
        err = float((p.grad - q.grad).norm() / (q.grad.norm() + 1e-12))
        assert err < 2e-2, (n, err)  # a missed or doubled micro-step would be off by a third or more


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (520, 384, 200), (2048, 2304, 768), (1000, 776, 1024)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("block_n", [-128, -256])
def test_gemm_two_sm(M, N, K, a_mn, b_mn, block_n):
    """2-SM (cta_group::2) tiles against the fp32 reference, including epilogues and split-K."""
    kf = _kf()
    torch.manual_seed(11)
    if (a_mn and M % 8) or (b_mn and N % 8):
        pytest.skip("MN-major operands need 16-byte aligned rows")
    a = (torch.randn(K, M) if a_mn else torch.randn(M, K)).to(DEV, torch.bfloat16)
    b = (torch.randn(K, N) if b_mn else torch.randn(N, K)).to(DEV, torch.bfloat16)
    out = kf.gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn, out_dtype=torch.float32, block_n=block_n)
    assert _rel(out, kf.gemm_ref(a, b, a_mn_major=a_mn, b_mn_major=b_mn)) < 1e-4
    bias = torch.randn(N, device=DEV)
    aux = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    g = kf.gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn, bias=bias, aux=aux, act=kf.ACT_GELU, block_n=block_n)
    rg, rpre = kf.gemm_ref(a, b, a_mn_major=a_mn, b_mn_major=b_mn, bias=bias, act=kf.ACT_GELU)
    assert _rel(g, rg) < 1e-2 and _rel(aux, rpre) < 1e-2


@pytest.mark.parametrize("n,r,c", [(3, 200, 136), (2, 768, 3072), (1, 520, 1000), (2, 2048, 512)])
@pytest.mark.parametrize("block_n", [0, 128, 256, -128, -256])
def test_gemm_symmetric(n, r, c, block_n):
    """Symmetric products (upper tiles computed, mirrored in the epilogue) against the fp32 reference.

    X X^T, and b A + c A A with A symmetric (the Newton-Schulz pair); the
    result must also be symmetric up to bf16 rounding of one product.
    """
    kf = _kf()
    torch.manual_seed(13)
    if block_n < 0 and r < 256:
        pytest.skip("2-SM tiles need 256 rows")
    X = (torch.randn(n, r, c, device=DEV) / c ** 0.5).bfloat16()
    A = kf.gemm(X, X, block_n=block_n, symmetric=True)
    ref = kf.gemm_ref(X, X)
    assert _rel(A, ref) < 1e-2
    assert float((A.float() - A.float().transpose(1, 2)).abs().max()) <= 2e-2 * float(ref.abs().max())
    As = ((A.float() + A.float().transpose(1, 2)) / 2).bfloat16()  # exactly symmetric operand
    B = kf.gemm(As, As, d=As, alpha=2.0, beta=-4.0, block_n=block_n, symmetric=True)
    refB = kf.gemm_ref(As, As, d=As, alpha=2.0, beta=-4.0)
    assert _rel(B, refB) < 1e-2
    # the plain GEMM on the same operands agrees
    Bp = kf.gemm(As, As, d=As, alpha=2.0, beta=-4.0, block_n=block_n)
    assert _rel(B, Bp.float()) < 1e-2


@pytest.mark.parametrize("group", [0, 3, 8, 64])
def test_gemm_grouped_tile_order(group):
    """The grouped tile order (tile columns taken G at a time) gives the same products, 1-SM and 2-SM, fp32 split."""
    kf = _kf()
    from koochak_b200.ops import native

    torch.manual_seed(14)
    native().gemm_set_group(group)
    try:
        for M, N, K, bn in [(1000, 776, 520, 128), (2304, 1536, 768, -256), (3072, 768, 4096, 0)]:
            a = torch.randn(K, M, device=DEV).bfloat16()
            b = torch.randn(K, N, device=DEV).bfloat16()
            out = kf.gemm(a, b, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32, block_n=bn)
            assert _rel(out, kf.gemm_ref(a, b, a_mn_major=True, b_mn_major=True)) < 1e-4, (M, N, K, bn)
            x = torch.randn(M, K, device=DEV).bfloat16()
            w = torch.randn(N, K, device=DEV).bfloat16()
            y = kf.gemm(x, w, block_n=bn)
            assert _rel(y, kf.gemm_ref(x, w)) < 1e-2, (M, N, K, bn)
    finally:
        native().gemm_set_group(-1)


@pytest.mark.parametrize("C", [768, 1024, 2048, 3072, 4096])
@pytest.mark.parametrize("M", [5, 333, 4099])
@pytest.mark.parametrize("xdtype,with_res", [(torch.float32, True), (torch.float32, False), (torch.bfloat16, True)])
@pytest.mark.parametrize("rms", [True, False])
def test_norm_backward_staged_rows(C, M, xdtype, with_res, rms):
    """LayerNorm / RMSNorm backward with rows staged by bulk copies (C = 768 ... 4096): dx (+ residual), its bf16
    copy, dgamma and dbeta against the fp32 autograd reference, for row counts below, near and far above the
    CTA count."""
    kf = _kf()
    torch.manual_seed(15)
    x = torch.randn(M, C, device=DEV).to(xdtype)
    w = torch.rand(C, device=DEV) + 0.5
    b = None if rms else torch.randn(C, device=DEV)
    _, mean, rstd = kf.norm_forward(x, w, b, 1e-5, rms=rms, out_dtype=torch.bfloat16)
    dy = torch.randn(M, C, device=DEV).bfloat16()
    dres = torch.randn(M, C, device=DEV).to(xdtype) if with_res else None
    dx, dw, db, lp = kf.norm_backward(dy, x, w, mean, rstd, rms=rms, dres=dres, dx_dtype=xdtype, want_lp=True)
    xr = x.float().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    br = None if rms else b.clone().requires_grad_(True)
    yr = kf.rms_norm_ref(xr, wr, 1e-5) if rms else kf.layer_norm_ref(xr, wr, br, 1e-5)
    yr.backward(dy.float())
    want = xr.grad + (dres.float() if with_res else 0.0)
    tol = 1e-3 if xdtype == torch.float32 else 1e-2
    assert _rel(dx, want) < tol
    assert _rel(lp, want) < 1e-2
    assert _rel(dw, wr.grad) < tol
    if not rms:
        assert _rel(db, br.grad) < tol


@pytest.mark.parametrize("M,N,dtype", [(16384, 768, torch.bfloat16), (16384, 3072, torch.bfloat16), (777, 300, torch.float16),
                                       (1000, 2304, torch.float32), (5, 8, torch.bfloat16)])
def test_bias_grad_two_pass(M, N, dtype):
    """Column sums (bias gradient) against fp32 torch: written, accumulated, and bitwise equal on a repeat."""
    kf = _kf()
    from koochak_b200.ops import native

    torch.manual_seed(16)
    g = torch.randn(M, N, device=DEV).to(dtype)
    ref = g.float().sum(0)
    a = kf.bias_grad(g)
    assert _rel(a, ref) < 1e-4
    assert torch.equal(a, kf.bias_grad(g))  # no atomics: the same bits every run
    acc = torch.ones(N, device=DEV)
    native().bias_grad(g, acc, True)
    assert _rel(acc, ref + 1.0) < 1e-4

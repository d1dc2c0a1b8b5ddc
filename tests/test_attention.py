"""Attention core (pmb_attention_forward / _backward) against float64 attention.

The kernels compute softmax(q k^T / 8) v with fp32 accumulation and round P
and dS to the input type before their products (as torch's fused attention
kernels do), so they are compared with a float64 evaluation on the same
rounded inputs under the 16-bit bar of 2e-2 relative to the largest
magnitude of each result; the row log-sum-exp is fp32 throughout (1e-4).
Planes are views of a packed [b, n, 3, h, 64] projection output and of
[b, n, h, 64] buffers, so the strided addressing is exercised too.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from pymsst_b200 import _native as nat

SCALE = 64 ** -0.5


@pytest.fixture(autouse=True)
def _no_wait_gave_up(request):
    """After every GPU test here: no bounded tensor-core wait ran out (a kernel that gave up would leave rows
    unwritten that the sampled comparisons might not visit)."""
    yield
    if request.node.get_closest_marker("gpu") is not None and torch.cuda.is_available():
        torch.cuda.synchronize()
        assert nat.library().pmb_umma_timeout(1) == 0


def _ref(q, k, v):
    s = torch.einsum("bhnd,bhmd->bhnm", q, k) * SCALE
    lse = torch.logsumexp(s, dim=-1)
    return torch.softmax(s, dim=-1) @ v, lse


def _rel(a, b, floor=1e-2):
    """Largest error relative to the largest reference magnitude (at least `floor`: dQ and dK are exactly zero
    for one-position sequences, where only rounding noise remains)."""
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(floor))


def _qkv(b, n, h, dtype, device, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    packed = (torch.randn(b, n, 3, h, 64, generator=g) * scale).to(dtype).to(device)
    return [packed[:, :, i].transpose(1, 2).requires_grad_() for i in range(3)]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [1, 5, 62, 64, 65, 129, 258])
def test_attention_matches_float64(cuda_device, n, dtype):
    from pymsst_b200.fused import AttentionFn

    b, h = 3, 2
    q, k, v = _qkv(b, n, h, dtype, cuda_device, seed=n, scale=1.5)
    o = AttentionFn.apply(q, k, v)
    assert o.shape == (b, h, n, 64) and o.dtype == dtype
    qd, kd, vd = (t.detach().double().requires_grad_() for t in (q, k, v))
    od, lsed = _ref(qd, kd, vd)
    assert _rel(o, od) < 2e-2
    lse = o.grad_fn.saved_tensors[4][:, :n].reshape(b, h, n)
    torch.testing.assert_close(lse.double(), lsed.detach(), rtol=1e-4, atol=1e-4)

    go = torch.randn(b, h, n, 64, generator=torch.Generator().manual_seed(7)).to(dtype).to(cuda_device)
    gq, gk, gv = torch.autograd.grad(o, (q, k, v), go)
    rq, rk, rv = torch.autograd.grad(od, (qd, kd, vd), go.double())
    for got, want in ((gq, rq), (gk, rk), (gv, rv)):
        assert got.dtype == dtype and got.shape == want.shape
        assert _rel(got, want) < 2e-2, _rel(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [62, 258])
def test_attention_agrees_with_sdpa(cuda_device, n):
    """Same inputs through torch's SDPA (bf16): both stay within the 16-bit bar of each other."""
    from pymsst_b200.fused import AttentionFn

    q, k, v = _qkv(4, n, 8, torch.bfloat16, cuda_device, seed=3)
    o = AttentionFn.apply(q, k, v)
    go = torch.randn_like(o)
    g_own = torch.autograd.grad(o, (q, k, v), go)
    o_ref = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    g_ref = torch.autograd.grad(o_ref, (q, k, v), go)
    assert _rel(o, o_ref) < 2e-2
    for a, r in zip(g_own, g_ref):
        assert _rel(a, r) < 3e-2


@pytest.mark.gpu
@pytest.mark.parametrize("n", [62, 200])
def test_attention_is_deterministic(cuda_device, n):
    from pymsst_b200.fused import AttentionFn

    q, k, v = _qkv(3, n, 4, torch.bfloat16, cuda_device, seed=11)
    o1 = AttentionFn.apply(q, k, v)
    o2 = AttentionFn.apply(q, k, v)
    assert torch.equal(o1, o2)
    go = torch.randn_like(o1)
    first = torch.autograd.grad(o1, (q, k, v), go)
    second = torch.autograd.grad(o2, (q, k, v), go)
    for a, b in zip(first, second):
        assert torch.equal(a, b)


@pytest.mark.gpu
def test_attention_many_items_per_cta(cuda_device):
    """More (sequence, head, query-block) items than resident CTAs: every CTA runs several items, so the barrier
    phases and the tensor-memory buffers run across item boundaries."""
    from pymsst_b200.fused import AttentionFn

    q, k, v = _qkv(300, 130, 8, torch.bfloat16, cuda_device, seed=13)
    with torch.no_grad():
        o = AttentionFn.apply(q, k, v)
    idx = [0, 1, 149, 298, 299]
    od, _ = _ref(*(t.detach()[idx].double() for t in (q, k, v)))
    assert _rel(o[idx], od) < 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("n", [62, 100])
def test_attention_backward_many_items_per_cta(cuda_device, n):
    """Short sequences take the one-pass backward (every key and query of a head in one item; two sequences per
    item up to 64 positions): more items than CTAs, an odd sequence count, gradients checked on a sample."""
    from pymsst_b200.fused import AttentionFn

    q, k, v = _qkv(301, n, 4, torch.bfloat16, cuda_device, seed=17)
    o = AttentionFn.apply(q, k, v)
    go = torch.randn(o.shape, generator=torch.Generator().manual_seed(3)).to(o.dtype).to(cuda_device)
    grads = torch.autograd.grad(o, (q, k, v), go)
    idx = [0, 1, 150, 299, 300]
    qd, kd, vd = (t.detach()[idx].double().requires_grad_() for t in (q, k, v))
    od, _ = _ref(qd, kd, vd)
    refs = torch.autograd.grad(od, (qd, kd, vd), go[idx].double())
    for got, want in zip(grads, refs):
        assert _rel(got[idx], want) < 2e-2, _rel(got[idx], want)


@pytest.mark.gpu
def test_attention_large_logits_stay_finite(cuda_device):
    """Scores far from zero (|s| ~ 100): the running-max softmax must not overflow."""
    from pymsst_b200.fused import AttentionFn

    q, k, v = _qkv(2, 130, 2, torch.bfloat16, cuda_device, seed=5, scale=4.0)
    o = AttentionFn.apply(q, k, v)
    od, _ = _ref(*(t.detach().double() for t in (q, k, v)))
    assert torch.isfinite(o).all()
    assert _rel(o, od) < 2e-2
    gq, gk, gv = torch.autograd.grad(o, (q, k, v), torch.randn_like(o))
    assert all(torch.isfinite(g).all() for g in (gq, gk, gv))


@pytest.mark.gpu
def test_model_attention_backends_agree(cuda_device):
    """The Attention module's own kernel and a library backend give the same block output."""
    from pymsst_b200.roformer import Attention, RotaryEmbedding

    torch.manual_seed(0)
    attn = Attention(192, heads=8, dim_head=64, rotary_embed=RotaryEmbedding(64)).to(cuda_device)
    x = torch.randn(6, 62, 192, device=cuda_device).to(torch.bfloat16)  # transformer inputs are 16-bit under AMP
    outs = {}
    for backend in ("pmb", "efficient"):
        attn.set_cuda_attention_backend(backend)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            outs[backend] = attn(x).float()
    assert _rel(outs["pmb"], outs["efficient"]) < 2e-2


# ------------------------------------------------------------- host side (CPU)
def _lib():
    try:
        return nat.library()
    except nat.FusedKernelUnavailable as e:  # pragma: no cover - library not built
        pytest.skip(str(e))


@pytest.mark.parametrize(
    "dtype, dim_head, message",
    [(nat.F32, 64, "bf16 or fp16"), (nat.BF16, 32, "dim_head must be 64")],
)
def test_attention_rejects_unsupported_arguments(dtype, dim_head, message):
    lib = _lib()
    strides = nat.i64_array([0] * 12)
    st = lib.pmb_attention_forward(None, None, None, None, None, 1, 8, 1, dim_head, strides, ctypes.c_float(0.125),
                                   dtype, None)
    assert st != 0 and message in lib.pmb_last_error().decode()


def test_attention_rejects_unaligned_strides():
    lib = _lib()
    # aligned fake addresses, a sequence stride that is not a multiple of 8 elements
    strides = nat.i64_array([1001, 512, 64] * 4)
    st = lib.pmb_attention_forward(4096, 4096, 4096, 4096, 4096, 2, 8, 1, 64, strides, ctypes.c_float(0.125),
                                   nat.BF16, None)
    assert st != 0 and "multiples of 8" in lib.pmb_last_error().decode()


def test_attention_rejects_overlapping_plane_order():
    """[b, h, n, 64]-ordered strides (position stride below heads * head stride) are refused by the C ABI;
    AttentionFn copies such tensors into a [b, n, h, 64] plane first."""
    lib = _lib()
    n, h = 8, 2
    strides = nat.i64_array([h * n * 64, 64, n * 64] * 4)  # (sequence, position, head) of a bhnd tensor
    st = lib.pmb_attention_forward(4096, 4096, 4096, 4096, 4096, 2, n, h, 64, strides, ctypes.c_float(0.125),
                                   nat.BF16, None)
    assert st != 0 and "must not overlap" in lib.pmb_last_error().decode()


def test_attention_backward_workspace_size():
    lib = _lib()
    assert lib.pmb_attention_backward_workspace_size(0, 8, 8) == 0
    assert lib.pmb_attention_row_pitch(65) == 68 and lib.pmb_attention_row_pitch(64) == 64
    assert lib.pmb_attention_backward_workspace_size(3, 65, 2) >= 3 * 2 * 68 * 4


def test_set_cuda_attention_backend_hook():
    """The reference's training module calls set_cuda_attention_backend on every module that has it and fails
    when none does (src/pymsst/training/module.py:416-425)."""
    from pymsst_b200.roformer import ATTENTION_BACKENDS, BSRoformer

    model = BSRoformer(dim=32, depth=1, stereo=True, time_transformer_depth=1, freq_transformer_depth=1)
    setters = [m for m in model.modules() if getattr(m, "set_cuda_attention_backend", None) is not None]
    assert setters
    for name in ATTENTION_BACKENDS:
        for m in setters:
            m.set_cuda_attention_backend(name)
    with pytest.raises(ValueError):
        setters[0].set_cuda_attention_backend("bogus")


@pytest.mark.gpu
def test_partial_rotary_tables_are_rejected(cuda_device):
    """The fused projection rotates whole heads; a shorter angle table is refused, not read past its end."""
    from pymsst_b200.roformer import Attention, RotaryEmbedding

    attn = Attention(192, heads=8, dim_head=64, rotary_embed=RotaryEmbedding(32)).to(cuda_device)
    with pytest.raises(ValueError, match="angle tables"):
        attn(torch.randn(2, 62, 192, device=cuda_device).to(torch.bfloat16))

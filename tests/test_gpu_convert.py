"""f32 inputs under 16-bit autocast: frsa_convert_in / frsa_convert_out through
the C ABI against their definitions in fp32 torch (the reference's pair
rotation, fa_rope_full .py:177-179, and its transpose), then the whole
autocast path against the float64 oracle."""
import numpy as np
import pytest
import torch

from helpers import seeded_inputs

pytestmark = pytest.mark.gpu


def _tables(cs, N, D, has_cls):
    off = 1 if has_cls else 0
    c = torch.ones(N, D // 2, device="cuda")
    s = torch.zeros(N, D // 2, device="cuda")
    c[off:], s[off:] = cs.COSP[: N - off], cs.SINP[: N - off]
    return c, s


def _args(src, dst, cs, has_cls, dtype):
    from triton_fused_rope_flash_attn_b200 import _lib
    B, H, N, D = src[0].shape
    a = _lib.FrsaConvertArgs()
    a.q, a.k, a.v = (t.data_ptr() for t in src)
    a.q_out, a.k_out, a.v_out = (t.data_ptr() for t in dst)
    a.cosp, a.sinp = cs.COSP.data_ptr(), cs.SINP.data_ptr()
    a.B, a.H, a.N, a.D, a.n_pos = B, H, N, D, cs.COSP.shape[0]
    a.has_cls = int(has_cls)
    a.dtype = _lib.FRSA_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.FRSA_DTYPE_F16
    return a


@pytest.mark.parametrize("B,H,side,has_cls,D,dtype", [(2, 3, 14, True, 64, torch.bfloat16),
                                                      (1, 2, 7, False, 80, torch.float16)])
def test_convert_kernels_match_torch(B, H, side, has_cls, D, dtype):
    from triton_fused_rope_flash_attn_b200 import CosSinTable, _lib
    N = side * side + (1 if has_cls else 0)
    cs = CosSinTable(100.0, side, D, device="cuda")
    c, s = _tables(cs, N, D, has_cls)
    g = torch.Generator(device="cuda").manual_seed(5)
    src = [torch.randn(B, H, N, D, device="cuda", generator=g) for _ in range(3)]
    dst = [torch.empty(B, H, N, D, device="cuda", dtype=dtype) for _ in range(3)]
    assert _lib.load().frsa_convert_in(_args(src, dst, cs, has_cls, dtype), None) == 0
    back = [torch.empty(B, H, N, D, device="cuda") for _ in range(3)]
    assert _lib.load().frsa_convert_out(_args(dst, back, cs, has_cls, dtype), None) == 0
    torch.cuda.synchronize()

    def rot(t, sign):
        e, o = t[..., 0::2], t[..., 1::2]
        return torch.stack((e * c - sign * o * s, o * c + sign * e * s), dim=-1).flatten(-2)

    want_in = [rot(src[0], 1), rot(src[1], 1), src[2]]
    for got, want in zip(dst, want_in):
        err = (got.float() - want).abs().max().item()
        assert err <= 2 ** -7 * want.abs().max().item(), err
    want_out = [rot(dst[0].float(), -1), rot(dst[1].float(), -1), dst[2].float()]
    for got, want in zip(back, want_out):
        assert (got - want).abs().max().item() <= 1e-5 * want.abs().max().item()
    # R^T R = I: converting in and back out returns the inputs to 16-bit rounding.
    for got, want in zip(back, src):
        assert (got - want).abs().max().item() <= 2 ** -7 * want.abs().max().item()


def test_autocast_f32_path_against_oracle():
    """sdpa_triton_fa_rope with f32 leaves under bf16 autocast (the reference
    README's usage) against the float64 oracle on the same
    f32 inputs, with the north-star bar (max 3e-2, mean 1e-3)."""
    from oracle import attn_bwd_np, attn_fwd_np
    from triton_fused_rope_flash_attn_b200 import CosSinTable, sdpa_triton_fa_rope
    B, H, side, has_cls, D = 2, 3, 16, True, 64   # N = 257: the general kernels
    N = side * side + 1
    q, k, v, do = seeded_inputs(B, H, N, D, 1.0, 7)
    cs = CosSinTable(100.0, side, D, device="cuda")
    leaves = [t.cuda().float().requires_grad_(True) for t in (q, k, v)]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        o = sdpa_triton_fa_rope(*leaves, cs, has_cls=has_cls, H_img=side)
    assert o.dtype == torch.float32
    o.backward(do.cuda().float())
    torch.cuda.synchronize()
    cos, sin = cs.COSP.cpu().numpy(), cs.SINP.cpu().numpy()
    qn, kn, vn, don = (t.double().numpy() for t in (q, k, v, do))
    o_ref, _ = attn_fwd_np(qn, kn, vn, cos, sin, has_cls)
    refs = (o_ref,) + attn_bwd_np(qn, kn, vn, don, cos, sin, has_cls)
    for got, ref in zip((o, leaves[0].grad, leaves[1].grad, leaves[2].grad), refs):
        d = np.abs(got.detach().double().cpu().numpy() - ref)
        assert d.max() <= 3e-2 and d.mean() <= 1e-3, (d.max(), d.mean())

"""LayerNorm + input projections on the tensor cores (eacs_project) against a
float32 PyTorch restatement of the reference's autocast path
(cst_ssm/modules/eacs.py:334 / :376 and :261-267), and against exact
(float64) arithmetic on the same rounded weights.

The restatement rounds where autocast rounds: LayerNorm in float32, its output
to the GEMM type T, the bias to T, the float32 sum of products plus bias to
T.  The kernel forms LayerNorm's statistics and the sums of products in other
orders, so a LayerNorm value that sits next to a rounding boundary of T can
round the other way, and a result can land on the neighbouring T value.  The
checks: (1) at least 99.9% of the elements within 2 units in the last place
of T of the restatement (2^-7 relative for bfloat16, 2^-10 for float16, or
1e-4 of the largest output where the sum cancels); (2) against float64
arithmetic the kernel is as accurate as the restatement: its largest error
at most 1.5x, its mean error at most 1.2x the restatement's.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _modules(d, H, N, seed):
    torch.manual_seed(seed)
    norm = torch.nn.LayerNorm(d).to(DEV)
    with torch.no_grad():
        norm.weight.uniform_(0.5, 1.5)
        norm.bias.uniform_(-0.2, 0.2)
    return norm, torch.nn.Linear(d, H).to(DEV), torch.nn.Linear(d, 2 * N).to(DEV), torch.nn.Linear(d, 2 * N).to(DEV)


def _restated(x, norm, pu, pb, pc, T, exact=False):
    torch.backends.cuda.matmul.allow_tf32 = False
    ft = torch.float64 if exact else torch.float32
    xn = torch.nn.functional.layer_norm(x.to(ft), (x.shape[-1],), norm.weight.to(ft), norm.bias.to(ft), norm.eps)
    xn = xn if exact else xn.to(T).to(ft)
    out = []
    for lin in (pu, pb, pc):
        acc = xn @ lin.weight.to(T).to(ft).T + lin.bias.to(T).to(ft)
        out.append(acc if exact else acc.to(T).to(ft))
    N = pb.weight.shape[0] // 2
    u, b, c = (o.detach() for o in out)
    return u, torch.complex(b[..., :N], b[..., N:]), torch.complex(c[..., :N], c[..., N:])


def _close(got, ref, exact, T):
    ulp = 2.0 ** -7 if T == torch.bfloat16 else 2.0 ** -10
    got, ref, exact = got.double(), ref.double(), exact.double()
    err = (got - ref).abs()
    floor = 1e-4 * float(ref.abs().max())
    near = (err <= 2 * ulp * ref.abs() + floor).double().mean()
    assert float(near) >= 0.999, float(near)
    e_got, e_ref = (got - exact).abs(), (ref - exact).abs()
    assert float(e_got.max()) <= 1.5 * float(e_ref.max()) + 1e-7, (float(e_got.max()), float(e_ref.max()))
    assert float(e_got.mean()) <= 1.2 * float(e_ref.mean()) + 1e-9, (float(e_got.mean()), float(e_ref.mean()))


def _check(out, x, mods, T):
    u, Bc, Cc = out
    ref = _restated(x, *mods, T)
    ex = _restated(x, *mods, T, exact=True)
    _close(u.float(), ref[0], ex[0], T)
    for k in (1, 2):
        _close(torch.view_as_real(out[k]), torch.view_as_real(ref[k]), torch.view_as_real(ex[k]), T)


@pytest.mark.parametrize("M,d,H,N,x_dtype,T", [
    (300, 768, 768, 16, torch.float16, torch.float16),     # config 1's widths, ragged M
    (257, 768, 768, 16, torch.bfloat16, torch.bfloat16),
    (128, 64, 64, 4, torch.float16, torch.float16),        # one k-block
    (1000, 1024, 1024, 16, torch.bfloat16, torch.bfloat16),  # config 2's widths (1088 -> 1280 rows)
    (200, 200, 120, 8, torch.float32, torch.bfloat16),     # fp32 activations, ragged d (k-block tail)
])
def test_project_vs_restatement(M, d, H, N, x_dtype, T):
    from eacs_b200 import _lib
    from eacs_b200.ops.projection import project
    norm, pu, pb, pc = _modules(d, H, N, seed=M + d)
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(M, d, generator=g) * 1.5 + 0.3).to(DEV).to(x_dtype)
    n0 = _lib.kernel_launches()
    u, Bc, Cc = project(x, norm, pu, pb, pc, T)
    torch.cuda.synchronize()
    assert _lib.kernel_launches() > n0
    assert u.dtype == T and Bc.dtype == torch.complex64
    _check((u, Bc, Cc), x, (norm, pu, pb, pc), T)
    assert _lib.device_status() == 0


def test_project_config1_rows_and_u_dtypes():
    """Config 1's full projection (8 x 4096 rows, 768 -> 768 + 32 + 32) with
    u kept as float32 of the rounded values, as the cell consumes it."""
    from eacs_b200.ops.projection import project
    norm, pu, pb, pc = _modules(768, 768, 16, seed=1)
    x = torch.randn(8, 4096, 768, generator=torch.Generator().manual_seed(2)).to(DEV).half()
    u16, Bc, Cc = project(x, norm, pu, pb, pc, torch.float16)
    u32, Bc2, Cc2 = project(x, norm, pu, pb, pc, torch.float16, u_dtype=torch.float32)
    torch.cuda.synchronize()
    assert u32.dtype == torch.float32 and u16.shape == (8, 4096, 768)
    assert torch.equal(u16.float(), u32) and torch.equal(Bc, Bc2) and torch.equal(Cc, Cc2)
    _check((u32.reshape(-1, 768), Bc.reshape(-1, 16), Cc.reshape(-1, 16)), x.reshape(-1, 768),
           (norm, pu, pb, pc), torch.float16)

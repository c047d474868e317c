"""Host-side properties of the fp16-pair weight split (no GPU): per-column power-of-two
scales, hi + lo / 2^11 reconstructing the scaled weights to ~2^-22 of each column's largest
entry, and zero columns left unscaled."""
import torch

from tt_atom.engine import _split_f16


def test_f16_split_reconstructs_scaled_columns():
    g = torch.Generator().manual_seed(0)
    t = torch.randn(64, 200, generator=g) * torch.logspace(-12, 12, 64)[:, None]
    t[3] = 0.0
    hi, lo, inv = _split_f16(t)
    assert hi.dtype == torch.float16 and lo.dtype == torch.float16 and inv.dtype == torch.float32
    s = 1.0 / inv
    m, e = torch.frexp(s)
    assert torch.all(m == 0.5)                                  # powers of two
    scaled = (t * s[:, None]).double()
    mx = scaled.abs().amax(1)
    nz = mx > 0
    assert torch.all((mx[nz] >= 2.0 ** 14) & (mx[nz] < 2.0 ** 15))
    rec = hi.double() + lo.double() / 2048.0
    err = (rec - scaled).abs().amax(1)
    assert torch.all(err[nz] <= 2.0 ** -21 * mx[nz])
    assert inv[3] == 1.0 and torch.all(hi[3] == 0) and torch.all(lo[3] == 0)
    assert torch.isfinite(hi.float()).all() and torch.isfinite(lo.float()).all()

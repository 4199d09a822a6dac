"""The int8 256-wide slice GEMM at several full waves of tiles, against the
oracle on blocks of the same seeded inputs.

4096 x 8192 x 4096 gives 256 output tiles of 256 x 256 on 74 CTA pairs:
three full waves and a last wave of 34 tiles, which the pair split cuts into
chunks.  Rows of A and columns of B are extracted independently, so the
oracle's result on a block's rows and columns is exactly that block of the
full reference result.  Blocks are taken from the first tile, a middle tile
and the last tile (a split one).  Checked there:
  * accumulation='fused' (exact fixed-point sums): within the fixed-point
    resolution of the reference's FP64 pipeline element by element, and a
    normwise error against the exact product no worse than 1.5x the
    reference's own error on the same blocks;
  * accumulation='ondevice': the reference's fused result bit for bit.
The second case is the wide-range 'max' configuration (entries
(U(0,1)-0.5)*exp(10*N(0,1))) at the same size.
"""

import numpy as np
import pytest
import torch

import ozaki_oracle as O
from conftest import same_bits

pytestmark = pytest.mark.gpu

BLOCKS = [(0, 64, 0, 256), (2048, 2112, 1792, 2048), (4032, 4096, 3840, 4096)]


def _inputs(kind):
    rng = np.random.RandomState(0)
    n, k, m = 4096, 8192, 4096
    if kind == "normal":
        return rng.randn(n, k), rng.randn(k, m)
    A = (rng.rand(n, k) - 0.5) * np.exp(10 * rng.randn(n, k))
    B = (rng.rand(k, m) - 0.5) * np.exp(10 * rng.randn(k, m))
    return A, B


@pytest.mark.parametrize("kind,preset", [("normal", (4, 1)), ("wide", (5, 4))])
def test_multiwave_int8_gemm_against_oracle_blocks(kind, preset):
    from ozaki_jax_b200.matmul import _ondevice_device
    n_hi, n_lo = preset
    A, B = _inputs(kind)
    Ad, Bd = torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda()
    C, st = _ondevice_device(Ad, Bd, n_hi, n_lo, "fused")
    torch.cuda.synchronize()
    assert st.item() == 0
    C = C.cpu().numpy()
    n_pairs = n_hi * n_hi + 2 * n_hi * n_lo
    ours, ref_f, ref_n, exact = [], [], [], []
    for r0, r1, c0, c1 in BLOCKS:
        Ab, Bb = A[r0:r1], B[:, c0:c1]
        c = C[r0:r1, c0:c1]
        nb = O.ondevice_numpy(Ab, Bb, n_hi, n_lo)
        rmax = np.max(np.abs(Ab), axis=1)[:, None]
        cmax = np.max(np.abs(Bb), axis=0)[None, :]
        bound = n_pairs * 2.0 ** -48 * rmax * cmax + 64 * 2.0 ** -52 * (np.abs(Ab) @ np.abs(Bb))
        assert np.all(np.abs(c - nb) <= bound), (r0, c0)
        ours.append(c)
        ref_n.append(nb)
        ref_f.append(O.fused_ondevice(Ab, Bb, n_hi, n_lo)[2])
        exact.append(O.exact_product(Ab, Bb))
    cat = lambda xs: np.concatenate([x.ravel() for x in xs])
    E = cat(exact)
    e_ref = min(e for e in (O.rel_err(cat(ref_f), E), O.rel_err(cat(ref_n), E)) if np.isfinite(e))
    assert O.rel_err(cat(ours), E) <= max(1.5 * e_ref, 32 * 2.0 ** -52)

    # the reference's own accumulation, bit for bit
    del C
    C2, st = _ondevice_device(Ad, Bd, n_hi, n_lo, "ondevice")
    torch.cuda.synchronize()
    C2 = C2.cpu().numpy()
    for (r0, r1, c0, c1), f in zip(BLOCKS, ref_f):
        assert same_bits(C2[r0:r1, c0:c1], f), (r0, c0)

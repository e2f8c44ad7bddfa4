"""The thread-to-butterfly pairings that let a thread hold a bin and its mirror N - k.

Two kernels rely on them:
- the RoFormer fused kernel at n_fft 2048 (kernels.cu, the mirror step and MaskOp::bin): the
  forward plan 16-16-8 ends in radix-8 butterflies, thread t takes g0 = t and g1 = 256 - t
  (thread 0: 0 and 128), and the split, the mask, the repack and the inverse's first radix-8
  pass run in registers;
- the HTDemucs back kernel at n_fft 4096 (split.cu, lane pairs): threads 2m and 2m + 1 take the
  inverse's first radix-16 butterflies m and 256 - m (thread 1: 128) and swap the mirrored points
  with one shuffle.

These tests replay the kernels' index formulas in numpy (a Stockham pass reads j + r*N/R and
writes base + r*NS, fft.cuh: pass_io) against np.fft, so that a change of radix plan or of the
slot formulas that breaks a pairing fails here, on the CPU.
"""
import numpy as np


def dft_matrix(r, inv):
    m = np.arange(r)
    return np.exp((2j if inv else -2j) * np.pi * np.outer(m, m) / r)


def stockham_pass(x, r, ns, inv=False):
    """One pass of fft.cuh's Stockham autosort, all butterflies at once."""
    n = len(x)
    nb = n // r
    j = np.arange(nb)
    k = j % ns
    rr = np.arange(r)[:, None]
    v = x[j[None, :] + nb * rr]
    if ns > 1:
        v = v * np.exp((2j if inv else -2j) * np.pi * k[None, :] * rr / (ns * r))
    v = dft_matrix(r, inv) @ v
    out = np.empty_like(x)
    out[((j // ns) * ns * r + k)[None, :] + ns * rr] = v
    return out


def split_repack(x, xm, f, n, ml, mr, sc=0.5):
    """The kernels' channel split, a complex mask per channel, and the repack (kernels.cu)."""
    zl = complex(sc * (x.real + xm.real), sc * (x.imag - xm.imag))
    zr = complex(sc * (x.imag + xm.imag), -sc * (x.real - xm.real))
    yl, yr = zl * ml[f], zr * mr[f]
    if f in (0, n // 2):
        yl, yr = complex(yl.real, 0.0), complex(yr.real, 0.0)
    gx = complex(yl.real - yr.imag, yl.imag + yr.real)
    gm = complex(yl.real + yr.imag, yr.real - yl.imag)
    return gx, gm


def packed_reference(spec, n, ml, mr):
    g = np.zeros(n, complex)
    for f in range(n // 2 + 1):
        fm = 0 if f == 0 else n - f
        gx, gm = split_repack(spec[f], spec[fm], f, n, ml, mr)
        g[f] = gx
        if f not in (0, n // 2):
            g[fm] = gm
    return g


def roformer_bin(tid, i, n=2048):
    """MaskOp<ARCH_ROFORMER, 2048, 128>::bin."""
    if i < 4:
        return tid + 256 * i
    if i < 8:
        return (256 - tid if tid else 128) + 256 * (i - 4)
    return n // 2 if tid == 0 else n // 2 + 1


def test_roformer_bins_cover_every_bin_once():
    bins = [roformer_bin(t, i) for t in range(128) for i in range(9)]
    valid = sorted(f for f in bins if f <= 1024)
    assert valid == list(range(1025))


def test_roformer_mirror_step_matches_fft():
    n = 2048
    rng = np.random.default_rng(11)
    x = rng.standard_normal(n) + 1j * rng.standard_normal(n)
    ml = rng.standard_normal(n // 2 + 1) + 1j * rng.standard_normal(n // 2 + 1)
    mr = rng.standard_normal(n // 2 + 1) + 1j * rng.standard_normal(n // 2 + 1)
    spec = np.fft.fft(x)
    want = np.fft.ifft(packed_reference(spec, n, ml, mr)) * n

    d = stockham_pass(stockham_pass(x, 16, 1), 16, 16)      # the forward's passes before the step
    out = np.empty(n, complex)
    f8, i8 = dft_matrix(8, False), dft_matrix(8, True)
    tol = 1e-9 * np.abs(spec).max()
    for tid in range(128):
        t0 = tid == 0
        groups = (tid, 256 - tid if tid else 128)
        z = np.zeros(16, complex)
        for h, g in enumerate(groups):                     # the forward's last pass, radix 8
            v = d[g + 256 * np.arange(8)] * np.exp(-2j * np.pi * g * np.arange(8) / n)
            z[8 * h:8 * h + 8] = f8 @ v
        gx, gm = [0j] * 9, [0j] * 9
        for i in range(9):
            if not (i < 8 or t0):
                continue
            f = roformer_bin(tid, i)
            xx = z[i] if i < 4 else (z[i + 4] if i < 8 else z[4])
            xm = (z[(8 - i) & 7] if t0 else z[15 - i]) if i < 4 else \
                ((z[19 - i] if t0 else z[11 - i]) if i < 8 else z[4])
            assert abs(xx - spec[f]) < tol and abs(xm - spec[0 if f == 0 else n - f]) < tol
            gx[i], gm[i] = split_repack(xx, xm, f, n, ml, mr)
        for i in range(4):                                  # the scatter back (kernels.cu)
            z[i] = gx[i]
            z[i + 8] = gx[i + 4]
            z[12 + i] = gm[7 - i] if t0 else gm[3 - i]
        z[4] = gx[8] if t0 else gm[7]
        for m in range(1, 4):
            z[4 + m] = gm[4 - m] if t0 else gm[7 - m]
        for h, g in enumerate(groups):                     # the inverse's first pass, radix 8
            out[8 * g + np.arange(8)] = i8 @ z[8 * h:8 * h + 8]
    got = stockham_pass(stockham_pass(out, 16, 8, inv=True), 16, 128, inv=True)
    assert np.abs(got - want).max() <= 1e-10 * np.abs(want).max()


def test_htdemucs_lane_pairs_hold_the_first_pass_points():
    n, nb = 4096, 256
    rng = np.random.default_rng(12)
    ml = rng.standard_normal(n // 2 + 1) + 1j * rng.standard_normal(n // 2 + 1)
    mr = rng.standard_normal(n // 2 + 1) + 1j * rng.standard_normal(n // 2 + 1)
    # the back kernel repacks masked spectra loaded per bin: any spectrum does here
    spec = rng.standard_normal(n) + 1j * rng.standard_normal(n)
    want = packed_reference(spec, n, ml, mr)
    lanes = {}
    for tid in range(256):
        m2 = tid >> 1
        j = (nb - m2 if m2 else nb // 2) if tid & 1 else m2
        v, gm, g8 = [None] * 16, [0j] * 9, 0j
        for r in range(9):
            if r < 8 or tid == 0:
                f = j + nb * r
                fm = 0 if f == 0 else n - f
                gx, gmv = split_repack(spec[f], spec[fm], f, n, ml, mr)
                if r < 8:
                    v[r], gm[r] = gx, gmv
                else:
                    g8 = gx
        lanes[tid] = (j, v, gm, g8)
    assert sorted(j for j, *_ in lanes.values()) == list(range(nb))
    for tid, (j, v, gm, g8) in lanes.items():
        partner_gm = lanes[tid ^ 1][2]
        for r in range(8, 16):                              # the shuffle (split.cu)
            own = gm[15 - r] if tid == 1 else (g8 if r == 8 else gm[(16 - r) & 7])
            v[r] = partner_gm[15 - r] if tid > 1 else own
        assert np.allclose(v, want[j + nb * np.arange(16)], rtol=0, atol=1e-12)

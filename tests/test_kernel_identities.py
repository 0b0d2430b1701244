"""CPU checks of identities the fused kernels rely on (numpy, f64).

1. stft_tma_kernel (spectral_stft_tma.cuh) unpacks two real segments a, b
   from Z = FFT(w a / 2 + i w b / 2) in registers: thread t of a group runs
   last-pass (radix-8) butterfly j = 4 (t % 32) + t // 32 and its mirror
   256 - j (128 for j = 0), holding Z[j + 256 r] in register 8 h + bitrev8(r)
   (h = 0 for j, 1 for the mirror), and forms
       A[k] = Z[k] + conj Z[L-k],  B[k] = -i (Z[k] - conj Z[L-k])
   for its bins k = j + 256 r and (mirror) + 256 r, r = 0..3, plus bin 1024
   for t = 0.  A and B must be the FFTs of w a and w b.
2. accum_fast_kernel's csd / coherence cross products (spectral_accum_fast.cuh)
   use, for Zx = FFT(xa + i xb) and Zy = FFT(ya + i yb) with m = L - k:
       4 (conj(Xa) Ya + conj(Xb) Yb) = 2 (conj(Zx[k]) Zy[k] + Zx[m] conj(Zy[m]))
       4 (|Xa|^2 + |Xb|^2)          = 2 (|Zx[k]|^2 + |Zx[m]|^2)
   with the real and imaginary parts as the kernel writes them.
"""
import numpy as np


def _bitrev8(r):
    return int(f"{r:03b}"[::-1], 2)


def test_stft_mirrored_unpack_map():
    L = 2048
    rng = np.random.default_rng(7)
    a, b, w = rng.standard_normal(L), rng.standard_normal(L), rng.random(L)
    Z = np.fft.fft(0.5 * w * a + 0.5j * w * b)
    FA, FB = np.fft.fft(w * a), np.fft.fft(w * b)
    seen = []
    for t in range(128):
        wq, lane = t >> 5, t & 31
        jb0 = 4 * lane + wq
        jb1 = 128 if jb0 == 0 else 256 - jb0
        t0 = jb0 == 0
        v = np.zeros(16, complex)
        for r in range(8):
            v[_bitrev8(r)] = Z[jb0 + 256 * r]
            v[8 + _bitrev8(r)] = Z[jb1 + 256 * r]
        for r in range(4):
            zk1 = v[_bitrev8(r)]
            zm1 = v[_bitrev8((8 - r) & 7)] if t0 else v[8 + _bitrev8(7 - r)]
            zk2 = v[8 + _bitrev8(r)]
            zm2 = v[8 + _bitrev8(7 - r)] if t0 else v[_bitrev8(7 - r)]
            for zk, zm, k in ((zk1, zm1, jb0 + 256 * r), (zk2, zm2, jb1 + 256 * r)):
                A = complex(zk.real + zm.real, zk.imag - zm.imag)
                B = complex(zk.imag + zm.imag, zm.real - zk.real)
                assert abs(A - FA[k]) < 1e-9 * abs(FA).max()
                assert abs(B - FB[k]) < 1e-9 * abs(FB).max()
                seen.append(k)
        if t0:
            z = v[_bitrev8(4)]
            assert abs(complex(2 * z.real, 0) - FA[1024]) < 1e-9 * abs(FA).max()
            assert abs(complex(2 * z.imag, 0) - FB[1024]) < 1e-9 * abs(FB).max()
            seen.append(1024)
    assert sorted(seen) == list(range(L // 2 + 1))


def test_cross_products_without_unpacking():
    L = 256
    rng = np.random.default_rng(11)
    xa, xb, ya, yb = (rng.standard_normal(L) for _ in range(4))
    Zx, Zy = np.fft.fft(xa + 1j * xb), np.fft.fft(ya + 1j * yb)
    Xa, Xb, Ya, Yb = (np.fft.fft(s) for s in (xa, xb, ya, yb))
    scale = max(abs(Zx).max(), abs(Zy).max()) ** 2
    for k in range(L // 2 + 1):
        m = (L - k) % L
        xk, xm, yk, ym = Zx[k], Zx[m], Zy[k], Zy[m]
        re = 2 * (xk.real * yk.real + xk.imag * yk.imag
                  + xm.real * ym.real + xm.imag * ym.imag)
        im = 2 * (xk.real * yk.imag - xk.imag * yk.real
                  + xm.imag * ym.real - xm.real * ym.imag)
        ref = 4 * (np.conj(Xa[k]) * Ya[k] + np.conj(Xb[k]) * Yb[k])
        assert abs(re - ref.real) < 1e-12 * scale
        assert abs(im - ref.imag) < 1e-12 * scale
        sxx = 2 * (abs(xk) ** 2 + abs(xm) ** 2)
        assert abs(sxx - 4 * (abs(Xa[k]) ** 2 + abs(Xb[k]) ** 2)) < 1e-12 * scale

"""CPU check of the code rule the device packer (csrc/pack.cu) uses in place
of a division: code 2 iff w > RD_f32(|s| * (0.5 + 2^-25)), code 0 iff
w < -that (sign of w flipped for a negative scale), else 1.  Restated here
in numpy and compared with quantize.py's own arithmetic (torch's IEEE f32
division, round half to even, clamp; quantize.py:18-22) on weights placed
within a few ulps of +-scale/2 over scales of every magnitude and sign."""
import numpy as np
import torch

TIE = np.float64(0.5) + np.float64(2.0) ** -25


def threshold_codes(w: np.ndarray, s: np.ndarray) -> np.ndarray:
    w = w.astype(np.float32)
    s = s.astype(np.float32)
    t = np.abs(s).astype(np.float64) * TIE              # exact in double
    f = t.astype(np.float32)
    f = np.where(f.astype(np.float64) > t, np.nextafter(f, np.float32(-np.inf)), f)   # RD_f32
    x = np.where(np.signbit(s)[:, None], -w, w)
    with np.errstate(invalid="ignore"):
        return np.where(np.abs(x) > f[:, None], np.where(np.signbit(x), 0, 2), 1)


def reference_codes(w: np.ndarray, s: np.ndarray) -> np.ndarray:
    q = torch.round(torch.from_numpy(w) / torch.from_numpy(s)[:, None])
    return (torch.clamp(q, -1, 1).to(torch.int32) + 1).numpy() & 3


def boundary_case(rng, R=64, N=256):
    s = (np.exp(rng.uniform(-40, 40, R)) * rng.choice([-1, 1], R)).astype(np.float32)
    s[:4] = np.array([0.0, -0.0, np.inf, 1e-45], np.float32)
    half = s * np.float32(0.5)
    w = np.empty((R, N), np.float32)
    for j in range(N):
        k = int(rng.integers(-6, 7))
        v = half.copy()
        for _ in range(abs(k)):
            v = np.nextafter(v, np.float32(np.inf) if k > 0 else np.float32(-np.inf))
        w[:, j] = v * np.float32(rng.choice([-1, 1]))
    w[:, :8] = rng.normal(0, 1, (R, 8)).astype(np.float32) * np.abs(s)[:, None]
    w[0, 0], w[1, 1], w[2, 2] = np.nan, np.inf, -np.inf
    return w, s


def test_threshold_rule_matches_division_and_rounding():
    rng = np.random.default_rng(3)
    for _ in range(20):
        w, s = boundary_case(rng)
        assert np.array_equal(threshold_codes(w, s), reference_codes(w, s))


def test_threshold_rule_on_quantize_py_edges():
    # the rounding edges of the committed fixture rows, scale 1 and -1
    w = np.array([[0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 0.49999997, -0.49999997,
                   0.50000006, -0.50000006, 1.0, -1.0, 0.0, -0.0, 7.0, -7.0]], np.float32)
    for sc in (1.0, -1.0, 3.0e-39):
        s = np.array([sc], np.float32)
        assert np.array_equal(threshold_codes(w, s), reference_codes(w, s))

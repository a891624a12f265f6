"""The device softplus (softplus.cuh) emulated in float32 on the CPU: its
polynomial log1p and the max(z,0)+log1p(e^-|z|) form stay within 6e-5
(relative) of the float64 softplus (threshold 20) over the whole fp32 range that matters."""
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
HDR = os.path.join(os.path.dirname(HERE), "mlp_megakernel_b200", "csrc", "softplus.cuh")


def _coeffs():
    txt = open(HDR).read()
    c = {int(k): float(v) for k, v in re.findall(r"kSpC(\d) = (-?[0-9.eE+-]+)f;", txt)}
    return [c[i] for i in range(0, 5)]


def _device_softplus_f32(z):
    """float32 model of softplus_x2: e = 2^(-|z*log2e|), q by Horner (FFMA),
    h = fma(q, e, max(z, 0)) (one rounding)."""
    z = z.astype(np.float32)
    c = [np.float32(v) for v in _coeffs()]
    s = (z * np.float32(1.4426950408889634)).astype(np.float32)
    # ex2.approx has ~2^-22 relative error; model it with the exact value
    e = np.exp2(-np.abs(s).astype(np.float64)).astype(np.float32)
    q = c[4]
    for k in (3, 2, 1, 0):
        q = (q.astype(np.float64) * e + c[k]).astype(np.float32) if hasattr(q, "astype") else \
            np.float32(np.float64(q) * e.astype(np.float64) + c[k])
    h = q.astype(np.float64) * e.astype(np.float64) + np.maximum(z, np.float32(0)).astype(np.float64)
    return h.astype(np.float32)


def _softplus_f64(z):
    z = z.astype(np.float64)
    return np.where(z > 20, z, np.log1p(np.exp(np.minimum(z, 20))))


def test_coefficients_parse():
    assert len(_coeffs()) == 5


def test_softplus_poly_accuracy():
    z = np.concatenate([np.linspace(-40, 40, 400001), np.linspace(-1, 1, 100001),
                        np.array([0.0, 19.99, 20.0, 20.01, -88.0, 88.0])]).astype(np.float32)
    got = _device_softplus_f32(z).astype(np.float64)
    ref = _softplus_f64(z)
    err = np.abs(got - ref)
    # relative error below 6e-5 (plus fp32 rounding of the sum)
    tol = 6e-5 * np.abs(ref) + 2 * np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    assert (err <= tol).all(), (err / np.maximum(ref, 1e-30)).max()


def test_softplus_poly_below_fp16_resolution():
    """The error is well below half an fp16 ulp of h, so the fp16 operand fed to
    the next GEMM is mostly (about 97%) the same as with an exact softplus."""
    z = np.linspace(-8, 8, 200001).astype(np.float32)
    got = _device_softplus_f32(z).astype(np.float16)
    ref = _softplus_f64(z).astype(np.float16)
    assert np.mean(got != ref) < 0.05
    # and where they differ, by one fp16 ulp at most
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    assert (d <= np.spacing(ref.astype(np.float16)).astype(np.float64) * 1.01).all()

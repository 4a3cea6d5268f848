"""Shared test helpers: tolerance checks and seeded inputs."""
import numpy as np

# The north-star contract against the reference's fp32 path.
MAX_ABS = 2e-3
REL_L2 = 1e-3


def rel_l2(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))


def assert_close(got, want, max_abs=MAX_ABS, rel=REL_L2, what=""):
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = float(np.abs(got - want).max()) if got.size else 0.0
    r = rel_l2(got, want)
    assert err <= max_abs and r <= rel, f"{what}: max abs {err:.3e} (<= {max_abs}), rel L2 {r:.3e} (<= {rel})"
    return err, r


def delta_inputs(seed, T, hk, hv, d):
    """Config-3 style inputs: q,k ~ N(0,1) L2-normalised per head, q /= sqrt(d);
    v ~ N(0,1); beta = sigmoid(N(0,1)); gate = -softplus(N(0,1))."""
    import oracle

    q = oracle.l2_normalize(oracle.normal(seed, 1, T * hk * d).reshape(T, hk, d)) * np.float32(1 / np.sqrt(d))
    k = oracle.l2_normalize(oracle.normal(seed, 2, T * hk * d).reshape(T, hk, d))
    v = oracle.normal(seed, 3, T * hv * d).reshape(T, hv, d)
    a = oracle.normal(seed, 4, T * hv).astype(np.float64)
    g = (-np.where(a > 20, a, np.log1p(np.exp(a)))).astype(np.float32).reshape(T, hv)
    b = (1.0 / (1.0 + np.exp(-oracle.normal(seed, 5, T * hv).astype(np.float64)))).astype(np.float32).reshape(T, hv)
    return q.astype(np.float32), k.astype(np.float32), v, g, b


def load_attn_fixture(path):
    """A golden attention fixture with its inputs decoded to the fp32 values the reference used."""
    import oracle

    z = dict(np.load(path))
    dec = oracle.from_bf16_bits if str(z["dtype"]) == "bf16" else oracle.from_fp16_bits
    for name in ("k", "v", "q"):
        z[name] = dec(z[name + "_bits"]).reshape(z[name + "_bits"].shape)
    return z

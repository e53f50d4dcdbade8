"""Shared helpers for the parity tests: seeded graphs with the edge cases the
reference's code paths distinguish (isolated nodes, duplicate edges,
self-loops, hubs that take the heavy-row schedule)."""
import numpy as np

RTOL = 1e-5  # the parity bar for f32 layer outputs: |gpu - ref| <= 1e-6 + 1e-5 |ref|
ATOL = 1e-6


def rand_graph(n, e, seed, hub_deg=0, loops=0, dup=0):
    rng = np.random.default_rng(seed)
    src = rng.integers(0, n, e, dtype=np.int64)
    dst = rng.integers(0, n, e, dtype=np.int64)
    if n > 3:
        # keep the last node isolated
        src[src == n - 1] = 0
        dst[dst == n - 1] = 1 % (n - 1)
    parts_s, parts_d = [src], [dst]
    if hub_deg:
        parts_s.append(rng.integers(0, max(n - 1, 1), hub_deg))
        parts_d.append(np.full(hub_deg, 2 % n))
    if loops:
        v = rng.integers(0, max(n - 1, 1), loops)
        parts_s.append(v)
        parts_d.append(v)
    if dup and e:
        k = rng.integers(0, e, dup)
        parts_s.append(src[k])
        parts_d.append(dst[k])
    s = np.concatenate(parts_s)
    d = np.concatenate(parts_d)
    perm = rng.permutation(s.size)
    s, d = s[perm], d[perm]
    return np.concatenate([s, d]).astype(np.uint32), int(s.size)


def loopless(n, e, seed):
    rng = np.random.default_rng(seed)
    s = rng.integers(0, n, e)
    d = (s + 1 + rng.integers(0, n - 1, e)) % n
    return np.concatenate([s, d]).astype(np.uint32), e


def bits(a):
    return np.ascontiguousarray(np.asarray(a, np.float32)).view(np.uint32)


def assert_bits_equal(got, want, what=""):
    g, w = bits(got).ravel(), bits(want).ravel()
    assert g.shape == w.shape, what
    # NaN payloads differ between CPU and GPU; any NaN matches any NaN
    nan = np.isnan(np.asarray(got, np.float32).ravel()) & np.isnan(np.asarray(want, np.float32).ravel())
    bad = np.flatnonzero((g != w) & ~nan)
    if bad.size:
        i = bad[0]
        raise AssertionError(
            f"{what}: {bad.size} of {g.size} elements differ; first at {i}: "
            f"got {np.asarray(got).ravel()[i]!r} want {np.asarray(want).ravel()[i]!r}")


def assert_close(got, want, what="", rtol=RTOL, atol=ATOL):
    g = np.asarray(got, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    assert g.shape == w.shape, what
    both_nan = np.isnan(g) & np.isnan(w)
    err = np.abs(g - w)
    ok = (err <= atol + rtol * np.abs(w)) | both_nan | (g == w)
    if not ok.all():
        i = np.flatnonzero(~ok)[0]
        raise AssertionError(f"{what}: {int((~ok).sum())} of {g.size} outside tolerance; "
                             f"first at {i}: got {g[i]!r} want {w[i]!r}")

"""The shared-memory ring k-buffer of the render kernels (gf_render.cuh)
reproduces the reference's register network (gutKBufferRenderer.cuh:132-147)
exactly, ties included.  Both are modelled here in Python on random hit
streams with many equal hit distances; the sequences of composited hits must
be identical."""

import numpy as np
import pytest


def network_stream(hits, k):
    """Reference: kb[0..k) sorted ascending, compare-and-swap from the top;
    when full, kb[0] is composited and its distance set to -1 first."""
    kb = [(-1.0, None)] * k
    n = 0
    out = []
    for h in hits:
        if n == k:
            out.append(kb[0])
            kb[0] = (-1.0, kb[0][1])
        else:
            n += 1
        carry = h
        for i in range(k - 1, -1, -1):
            if carry[0] > kb[i][0]:
                kb[i], carry = carry, kb[i]
    out.extend(kb[k - n:])
    return out


def ring_stream(hits, k):
    """The ring: sorted list, pop the front when full, then insert by the
    closed-form rule (entries >= hit stay above it; below it, each run of
    equal distances moves its top entry to its bottom)."""
    buf = []
    ties = 0
    out = []
    for h in hits:
        if len(buf) == k:
            front = buf.pop(0)
            if buf and buf[0][0] == front[0]:
                ties -= 1
            out.append(front)
        if ties == 0:
            p = len(buf)
            while p > 0 and buf[p - 1][0] >= h[0]:
                p -= 1
        else:
            p = 0
            while p < len(buf) and buf[p][0] < h[0]:
                p += 1
            r = 0
            while r < p:
                e = r + 1
                while e < p and buf[e][0] == buf[r][0]:
                    e += 1
                if e - r >= 2:
                    top = buf.pop(e - 1)
                    buf.insert(r, top)
                r = e
        buf.insert(p, h)
        if p + 1 < len(buf) and buf[p + 1][0] == h[0]:
            ties += 1
    out.extend(buf)
    return out


@pytest.mark.parametrize("k", [1, 2, 4, 12, 16, 32])
@pytest.mark.parametrize("levels", [3, 8, 1000])
def test_ring_matches_network(k, levels):
    rng = np.random.default_rng(k * 1000 + levels)
    for trial in range(60):
        n = int(rng.integers(0, 3 * k + 10))
        # few distinct distances -> many exact ties; mostly increasing streams
        base = np.sort(rng.integers(0, levels, n)).astype(float)
        noise = rng.integers(-2, 3, n) * (rng.random(n) < 0.4)
        dist = np.clip(base + noise, 0, None) / 4.0
        hits = [(float(d), i) for i, d in enumerate(dist)]
        assert ring_stream(hits, k) == network_stream(hits, k), (k, levels, trial)


def test_ring_matches_the_reference_kbuffer():
    """The ring model against the reference's own HitParticleKBufferT
    (gutKBufferRenderer.cuh:118-166, compiled for the host:
    tests/golden/hit_golden.npz, made by tests/golden/make_hit_golden.py) on
    its recorded composite orders."""
    from pathlib import Path

    golden = np.load(Path(__file__).resolve().parent / "golden" / "hit_golden.npz")
    off = golden["kb_offsets"]
    for s, k in enumerate(golden["kb_k"]):
        t = golden["kb_hit_t"][off[s]:off[s + 1]]
        hits = [(float(d), i) for i, d in enumerate(t)]
        order = [i for _, i in ring_stream(hits, int(k))]
        assert order == golden["kb_order"][off[s]:off[s + 1]].tolist(), (s, int(k))

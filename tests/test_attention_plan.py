"""The decode attention's work split, restated on the CPU (no GPU needed).

attn_split_kernel (llama.rs_b200/csrc/decode.cu) cuts an item's context of L
positions into `nsplit` splits of `chunk` positions (a multiple of the
32-position tile, so a tile never straddles a 64-position KV page), runs an
online softmax over the split's tiles (running max and sum per head,
rescaling the accumulated PV), and merges the splits' (max, sum, o) with
exp(max_s - M) weights over the splits that saw positions.  This test
restates that dataflow in numpy, in the kernel's order, and checks it
against direct softmax attention (src/model.rs:206-231, softmax_inplace
:298-313) over ragged lengths, empty splits and every split count the host
can choose (1..64), so a change to the split arithmetic is caught without a
GPU.  The kernel itself is checked against the oracle by the GPU tests.
"""
import numpy as np
import pytest

TILE = 32
MIN_SPLIT = TILE


def split_chunk(L, nsplit):
    """Positions per split (decode.cu split_chunk)."""
    c = max((L + nsplit - 1) // nsplit, MIN_SPLIT)
    return (c + TILE - 1) & ~(TILE - 1)


def nsplit_for(sms, ctas_per_sm, batch, nkv, max_seq_len, max_split=64):
    """Split count of a step (capi.cu nsplit_for)."""
    want = 8 * sms * ctas_per_sm // (batch * nkv)
    maxs = max(1, (max_seq_len + 127) // 128)
    return max(1, min(want, max_split, maxs))


def kernel_attention(q, K, V, nsplit):
    """q: [G, hd] (already scaled), K/V: [L, hd].  Returns [G, hd]."""
    L = K.shape[0]
    G = q.shape[0]
    chunk = split_chunk(L, nsplit)
    parts = []
    for split in range(nsplit):
        s0, s1 = split * chunk, min(L, split * chunk + chunk)
        ntiles = (s1 - s0 + TILE - 1) // TILE if s0 < s1 else 0
        m = np.full(G, -np.inf, np.float32)
        lsum = np.zeros(G, np.float32)
        o = np.zeros((G, q.shape[1]), np.float32)
        for i in range(ntiles):
            t0 = s0 + TILE * i
            nv = min(TILE, s1 - t0)
            s = (q @ K[t0:t0 + nv].T).astype(np.float32)  # [G, nv]
            bm = s.max(axis=1)
            mn = np.maximum(m, bm)
            cf = np.where(m == -np.inf, 0.0, np.exp(m - mn)).astype(np.float32)
            e = np.exp(s - mn[:, None]).astype(np.float32)
            lsum = lsum * cf + e.sum(axis=1)
            m = mn
            o = o * cf[:, None] + e @ V[t0:t0 + nv]
        any_ = ntiles > 0
        parts.append((m if any_ else np.full(G, -np.inf, np.float32),
                      lsum if any_ else np.zeros(G, np.float32),
                      o if any_ else np.zeros_like(o)))
    nact = min(nsplit, (L + chunk - 1) // chunk)
    ms = np.stack([p[0] for p in parts[:nact]])        # [nact, G]
    M = ms.max(axis=0)
    w = np.where(ms == -np.inf, 0.0, np.exp(ms - M)).astype(np.float32)
    Ls = (np.stack([p[1] for p in parts[:nact]]) * w).sum(axis=0)
    O = (np.stack([p[2] for p in parts[:nact]]) * w[:, :, None]).sum(axis=0)
    # splits past nact saw no positions and carry (-inf, 0, 0)
    for p in parts[nact:]:
        assert np.all(p[0] == -np.inf) and np.all(p[1] == 0) and np.all(p[2] == 0)
    return O / Ls[:, None]


def direct_attention(q, K, V):
    s = q @ K.T
    p = np.exp(s - s.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    return p @ V


@pytest.mark.parametrize("L", [1, 2, 31, 32, 33, 63, 64, 65, 129, 1000, 1031, 1152, 2049])
@pytest.mark.parametrize("nsplit", [1, 2, 3, 9, 32, 64])
def test_split_tiles_and_merge_equal_softmax_attention(L, nsplit):
    rng = np.random.default_rng(L * 131 + nsplit)
    G, hd = 7, 128
    q = (rng.standard_normal((G, hd)) / np.sqrt(hd)).astype(np.float32)
    K = rng.standard_normal((L, hd)).astype(np.float32)
    V = rng.standard_normal((L, hd)).astype(np.float32)
    got = kernel_attention(q, K, V, nsplit)
    want = direct_attention(q.astype(np.float64), K.astype(np.float64), V.astype(np.float64))
    assert np.abs(got - want).max() < 2e-5


@pytest.mark.parametrize("L", [1, 33, 64, 1031, 4096])
@pytest.mark.parametrize("nsplit", [1, 7, 64])
def test_splits_cover_the_context_on_tile_and_page_boundaries(L, nsplit):
    chunk = split_chunk(L, nsplit)
    assert chunk % TILE == 0 and 64 % TILE == 0  # a tile never straddles a page
    covered = []
    for split in range(nsplit):
        s0, s1 = split * chunk, min(L, split * chunk + chunk)
        covered.extend(range(s0, s1))
    assert covered == list(range(L))  # every position once, in order
    assert nsplit * chunk >= L  # so the active splits are the first ceil(L / chunk)
    nact = min(nsplit, (L + chunk - 1) // chunk)
    assert nact == -(-L // chunk) and 1 <= nact <= 64  # the merge reads two partials per lane


def test_split_counts_of_the_benchmark_steps():
    # B200: 148 SMs, 3 attention CTAs per SM (f32 KV, head_dim 128)
    assert nsplit_for(148, 3, 64, 4, 4096) == 13   # c3, 64 sequences
    assert nsplit_for(148, 3, 1, 4, 4096) == 32    # c3, batch 1: 128 positions per split at full context
    assert nsplit_for(148, 3, 16, 8, 8192) == 27   # c4, 16 sequences
    for b in (1, 2, 8, 64, 256):
        n = nsplit_for(148, 3, b, 4, 4096)
        assert 1 <= n <= 64

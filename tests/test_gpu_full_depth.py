"""Full-depth parity on the benchmark configurations: the whole model, the
benchmark's prompt length and 128 greedy steps, against golden outputs of the
oracle's literal per-token scalar path (tests/golden/model_golden.py, which
made tests/golden/model_<case>.json).

* c3: Qwen2.5-7B shape, 28 layers, q4km, 1024-token prompt (attention past
  1000 positions, the tcgen05 prefill in 64-token chunks), 128 greedy steps.
* c2: Qwen2.5-1.5B shape, 28 layers, q4k (tied Q4_K head), 512-token prompt,
  128 greedy steps.

Bars: logits within 2e-2 max-abs at the stored indices (the oracle's top 64
and 1024 seeded random ones) after the prompt and after the last step, and
identical greedy tokens (on a mismatch the oracle's top-1/top-2 margin at
that step is reported).  The fixture records a SHA-256 of the model bytes; the
test rebuilds the model and checks it first.
"""
import json
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import model_golden  # noqa: E402

LOGIT_TOL = 2e-2


def _fixture(name):
    path = model_golden.fixture_path(name)
    if not os.path.exists(path):
        pytest.skip(f"fixture {os.path.basename(path)} not generated")
    with open(path) as f:
        return json.load(f)


def _logit_err(got, ref):
    idx = np.asarray(ref["index"])
    return float(np.abs(got[idx] - np.asarray(ref["value"], np.float32)).max())


@pytest.mark.parametrize("name", ["c2", "c3"])
@pytest.mark.parametrize("persistent", [False, True], ids=["graph", "persistent"])
def test_full_depth_greedy_matches_oracle(lrs, backend, name, persistent):
    fx = _fixture(name)
    cfg, sm, prompt, n_decode = model_golden.build(lrs, name, threads=os.cpu_count() or 1)
    assert model_golden.model_digest(sm.desc(), cfg) == fx["model_sha256"]
    assert len(prompt) == fx["prompt"] and n_decode == fx["decode"]
    model = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=len(prompt) + n_decode + 8,
                               persistent_decode=persistent)
    logits, first = model.prefill(prompt, 0)
    err0 = _logit_err(logits, fx["logits"]["0"])
    assert err0 < LOGIT_TOL, f"prefill logits max-abs error {err0}"
    assert first == fx["logits"]["0"]["argmax"]
    produced = model.decode_greedy([first], [len(prompt)], n_decode)[:, 0]
    fed = np.concatenate([[first], produced[:-1]]).astype(np.int64)
    want = np.asarray(fx["tokens"], np.int64)
    if not np.array_equal(fed, want):
        i = int(np.nonzero(fed != want)[0][0])
        raise AssertionError(f"greedy tokens diverge at step {i}: oracle {want[i]} gpu {fed[i]}; "
                             f"oracle top1-top2 margin there {fx['margins'][i]:.3e}")
    # logits after the last step: that step again (it rewrites the same KV row)
    last, am = model.forward_token(int(fed[-1]), len(prompt) + n_decode - 1)
    assert am == produced[-1]
    err1 = _logit_err(last, fx["logits"][str(n_decode)])
    assert err1 < LOGIT_TOL, f"final logits max-abs error {err1}"
    print(f"{name}: prefill err {err0:.2e}, final err {err1:.2e}, {n_decode} tokens match")
    model.close()

"""Tensor-parallel decode (the c4 layout) on 2 GPUs (4 for the uneven shards)
against the oracle.

Each rank is a separate process with its own GPU; rank 0 makes the NCCL id
and every rank passes the full model.  Bars: final logits within 2e-2 of the
oracle and identical greedy tokens, for one sequence and for a batch of three
(the batched matmul path), on every rank.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import assert_greedy

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import importlib.util, json, os, sys
root, rank, world, tp_id, out = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), bytes.fromhex(sys.argv[4]), sys.argv[5]
shape, recipe, p2p = json.loads(sys.argv[6]), sys.argv[7], sys.argv[8] == "p2p"
pkg = os.path.join(root, "llama.rs_b200")
spec = importlib.util.spec_from_file_location("llamars_b200", os.path.join(pkg, "__init__.py"),
                                              submodule_search_locations=[pkg])
lrs = importlib.util.module_from_spec(spec); sys.modules["llamars_b200"] = lrs; spec.loader.exec_module(lrs)
cfg = lrs.LlamaConfig(*shape)
sm = lrs.SynthModel(cfg, 11, lrs.LoadQuantization[recipe])
be = lrs.CudaBackend(rank)
m = lrs.CudaQwen2Model(be, sm.desc(), max_seq_len=256, max_sequences=4, tp_rank=rank,
                       tp_world=world, tp_id=tp_id, tp_p2p=p2p)
res = {}
prompt = lrs.prompt_tokens(11, 40, cfg.vocab_size)
logits, first = m.prefill(prompt, 0, seq=0)
res["logits"] = logits.tolist()
res["tokens"] = [int(first)] + m.decode_greedy([first], [40], 24, [0])[:, 0].tolist()
firsts = []
for s in range(1, 4):
    p = lrs.prompt_tokens(50 + s, 20 + s, cfg.vocab_size)
    firsts.append(int(m.prefill(p, 0, seq=s, want_logits=False)[1]))
prod = m.decode_greedy(firsts, [21, 22, 23], 16, [1, 2, 3])
res["batch"] = [[firsts[i]] + prod[:, i].tolist() for i in range(3)]
json.dump(res, open(out, "w"))
"""


SHAPES = {
    # hidden, intermediate, heads, kv heads, layers, vocab, eps, theta, ctx, head_dim, tied
    "aligned": ([512, 1024, 8, 4, 2, 2048, 1e-6, 1e6, 4096, 64, False], "Q4KM"),
    # o's and down's column shards are 2.5 and 5.5 Q4_K super-blocks wide: the
    # ranks hold the covering blocks and zero-pad x (the c4 layout at TP8)
    "windowed": ([1280, 2816, 10, 2, 2, 2048, 1e-6, 1e6, 4096, 128, False], "Q4K"),
    # at TP=4, o's shards are 1.75 super-blocks (the ranks cover 2 or 3) and
    # down's 2.75 (3 or 4): shards of one projection differ in width
    "uneven4": ([1792, 2816, 28, 4, 2, 2048, 1e-6, 1e6, 4096, 64, False], "Q4K"),
}
WORLD = {"uneven4": 4}


@pytest.mark.parametrize("shape", ["aligned", "windowed", "uneven4"])
@pytest.mark.parametrize("allreduce", ["nccl", "p2p"])
def test_tp2_matches_oracle(lrs, orc, tmp_path, allreduce, shape):
    """allreduce="p2p": the row-split projections are summed by the peer-memory
    all-reduce (the model option tp_p2p, tp_p2p.cu) instead of NCCL."""
    import torch
    world = WORLD.get(shape, 2)
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    dims, recipe = SHAPES[shape]
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0"}
    tp_id = lrs.tp_unique_id().hex()
    procs, outs = [], []
    for r in range(world):
        out = str(tmp_path / f"rank{r}.json")
        outs.append(out)
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER, ROOT, str(r), str(world), tp_id,
                                       out, json.dumps(dims), recipe, allreduce], env=env))
    try:
        codes = [p.wait(timeout=600) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert codes == [0] * world
    res = [json.load(open(o)) for o in outs]
    cfg = lrs.LlamaConfig(*dims)
    sm = lrs.SynthModel(cfg, 11, lrs.LoadQuantization[recipe])
    prompt = lrs.prompt_tokens(11, 40, cfg.vocab_size)
    ref = orc.OracleModel(sm.desc(), 256).benchmark_tokens(prompt, 25, keep_logits=True)
    for r in range(world):
        assert np.abs(np.array(res[r]["logits"], np.float32) - ref["logits"][0]).max() < 2e-2
        assert_greedy(ref, res[r]["tokens"])
        assert res[r]["batch"] == res[0]["batch"]
        assert res[r]["logits"] == res[0]["logits"]  # every rank holds the same residual
    for s in range(1, 4):
        p = lrs.prompt_tokens(50 + s, 20 + s, cfg.vocab_size)
        want = orc.OracleModel(sm.desc(), 256).benchmark_tokens(p, 17)
        assert_greedy(want, res[0]["batch"][s - 1])

"""Data-parallel host logic of bench.py on CPU: two gloo ranks share one
pre-quantized model file (rank 0 builds and writes it, rank 1 waits at the
barrier and maps it) and see identical bytes.  No GPU is used."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import hashlib, json, os, sys, ctypes
root, out = sys.argv[1], sys.argv[2]
sys.path.insert(0, root)
import torch.distributed as dist
import bench
dist.init_process_group("gloo")
rank = dist.get_rank()
lrs = bench.load_pkg()
wl = dict(bench.WORKLOADS["c0"], layers=1)
built_before = os.path.exists(bench.model_cache_path(wl))
cfg, mf = bench.build_model(lrs, wl, 2, dist.barrier, builder=rank == 0)
d = mf.desc().contents
h = hashlib.sha256()
for td in (d.embed_tokens, d.lm_head, d.layers[0].q_proj, d.layers[0].down_proj):
    h.update(ctypes.string_at(td.data, td.nbytes))
json.dump({"rank": rank, "sha": h.hexdigest(), "layers": cfg.num_hidden_layers,
           "tied": cfg.tie_word_embeddings, "built_before": built_before}, open(out, "w"))
dist.barrier()
dist.destroy_process_group()
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_share_one_model_file(tmp_path):
    port = _free_port()
    procs, outs = [], []
    for r in range(2):
        out = str(tmp_path / f"r{r}.json")
        outs.append(out)
        env = {**os.environ, "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(r),
               "WORLD_SIZE": "2", "TMPDIR": str(tmp_path)}
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER, ROOT, out], env=env))
    try:
        codes = [p.wait(timeout=300) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert codes == [0, 0]
    res = [json.load(open(o)) for o in outs]
    assert res[0]["sha"] == res[1]["sha"]
    assert res[0]["layers"] == res[1]["layers"] == 1
    assert res[0]["tied"] and res[1]["tied"]
    assert not res[0]["built_before"]
    assert len([f for f in os.listdir(tmp_path) if f.endswith(".lrs")]) == 1

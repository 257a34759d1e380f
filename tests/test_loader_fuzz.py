"""Corrupt model files against the loaders (CPU, no GPU needed).

GgufFile::open (src/gguf.rs:72-230), SafetensorStore / SafetensorsLoader
(src/loader.rs:80-230, 535-645) and ModelLoader::load return errors for a
bad file; so must the C ABI: every truncation and byte corruption below has
to end in success or an LrsError, never in a crash or an exception escaping
the library (a corrupt block count once asked for billions of layers).
Seeded, so every run tries the same files.
"""
import os
import random
import shutil

import pytest


def _cfg(lrs):
    return lrs.LlamaConfig(64, 128, 2, 1, 1, 100, 1e-6, 1e6, 256, 32, True)


def _try(fn):
    try:
        fn()
    except Exception as e:  # noqa: BLE001 -- only the library's own error type is allowed
        assert type(e).__name__ == "LrsError", repr(e)
        assert "\ufffd" not in str(e), str(e)  # the library's messages are UTF-8


@pytest.mark.parametrize("mode", ["truncate", "flip"])
def test_corrupt_gguf_files_fail_cleanly(lrs, tmp_path, mode):
    base = str(tmp_path / "base.gguf")
    sm = lrs.SynthModel(_cfg(lrs), 1, lrs.LoadQuantization.Q4KM)  # owns the description
    lrs.write_qwen2_gguf(base, sm.desc())
    data = open(base, "rb").read()
    path = str(tmp_path / "m.gguf")
    for k in range(300):
        rng = random.Random(k)
        b = bytearray(data)
        if mode == "truncate":
            b = b[:rng.randrange(0, len(b))]
        else:  # the header and tensor table: the first 4 KB
            for _ in range(rng.randrange(1, 8)):
                b[rng.randrange(0, min(len(b), 4096))] = rng.randrange(256)
        open(path, "wb").write(b)

        def load():
            g = lrs.GgufFile(path)
            try:
                g.qwen2_desc(lrs.LoadQuantization.NONE)
            finally:
                g.close()
        _try(load)


@pytest.mark.parametrize("mode", ["truncate", "flip", "config"])
def test_corrupt_safetensors_checkpoints_fail_cleanly(lrs, tmp_path, mode):
    base = tmp_path / "base"
    base.mkdir()
    sm = lrs.SynthModel(_cfg(lrs), 1, lrs.LoadQuantization.NONE)  # owns the description
    lrs.write_qwen2_safetensors(str(base), sm.desc(), dtype="BF16")
    stf = [f for f in sorted(os.listdir(base)) if f.endswith(".safetensors")][0]
    data = open(base / stf, "rb").read()
    cfg = open(base / "config.json", "rb").read()
    work = tmp_path / "work"
    shutil.copytree(base, work)
    hl = int.from_bytes(data[:8], "little") + 8
    for k in range(200):
        rng = random.Random(k)
        b, c = bytearray(data), bytearray(cfg)
        if mode == "truncate":
            b = b[:rng.randrange(0, len(b))]
        elif mode == "flip":  # the JSON header (and the first data bytes)
            for _ in range(rng.randrange(1, 6)):
                b[rng.randrange(0, min(len(b), hl + 64))] = rng.randrange(256)
        else:
            for _ in range(rng.randrange(1, 4)):
                c[rng.randrange(0, len(c))] = rng.randrange(256)
        open(work / stf, "wb").write(b)
        open(work / "config.json", "wb").write(c)
        for recipe in (lrs.LoadQuantization.NONE, lrs.LoadQuantization.Q4K):
            _try(lambda: lrs.LoadedModel(str(work), recipe).close())

"""The C host driver end to end on the GPU: KV-cached decode with the MoE
block in moe_ffn, against host_tiny.npz, which the reference's own
model_forward_f32 produced (recomputing the prefix at every step). Bar:
logits bit for bit at every step, identical greedy tokens."""
import os

import numpy as np
import pytest

from helpers import GOLDEN, TINY, model_records, tiny_model, write_bin

pytestmark = pytest.mark.gpu
mh = pytest.importorskip("moe_host")


def build(gpu, dt, base):
    g, attn, moe = tiny_model(dt, seed=1)
    m = mh.HostModel(TINY, batch=2, max_ctx=16, moe_base=base)
    m.set_globals(g["tok_emb"], g["final_norm_w"], g["lm_head"])
    for l, a in enumerate(attn):
        m.set_layer(l, a)
        gpu.upload_layer(base + l, moe[l])
    return m


@pytest.mark.parametrize("dt", [2, 3])
def test_host_decode_matches_reference_golden(gpu, dt):
    z = np.load(os.path.join(GOLDEN, "host_tiny.npz"))
    base = 500 + 10 * dt
    m = build(gpu, dt, base)
    toks = m.generate(z[f"prompt_{dt}"], 6)
    assert np.array_equal(toks, z[f"tokens_{dt}"])
    # teacher-forced: the logits of every step
    m.reset()
    logits = m.step(z[f"prompt_{dt}"])
    for s in range(6):
        assert np.array_equal(logits, z[f"logits_{dt}"][s]), f"step {s}"
        logits = m.step(z[f"tokens_{dt}"][:, s:s + 1])
    ms, calls, cpu = m.timing()
    assert list(calls) == [7 + 6] * TINY["n_layers"] and (ms > 0).all() and cpu > 0
    m.close()
    for l in range(TINY["n_layers"]):
        gpu.free_layer(base + l)


@pytest.mark.parametrize("dt", [2, 3])
def test_host_load_bin_matches_reference_golden(gpu, dt, tmp_path):
    z = np.load(os.path.join(GOLDEN, "host_tiny.npz"))
    g, attn, moe = tiny_model(dt, seed=1)
    p = str(tmp_path / "m.bin")
    write_bin(p, model_records(g, attn, moe))
    cfg = mh.config_from_bin(p)
    m = mh.HostModel(cfg, batch=2, max_ctx=16, moe_base=540 + 10 * dt)
    m.load_bin(p)
    assert np.array_equal(m.generate(z[f"prompt_{dt}"], 6), z[f"tokens_{dt}"])
    m.close()                                  # frees the model's resident MoE layers


def test_host_synth_deterministic(gpu):
    a = mh.HostModel(TINY, batch=2, max_ctx=24, moe_base=600)
    a.synth(7, 2)
    b = mh.HostModel(TINY, batch=2, max_ctx=24, moe_base=610)
    b.synth(7, 2)
    prompts = np.arange(10, dtype=np.int32).reshape(2, 5)
    ta, tb = a.generate(prompts, 8), b.generate(prompts, 8)
    assert np.array_equal(ta, tb) and ta.min() >= 0 and ta.max() < TINY["vocab_size"]
    # a prefilled context: decode continues from position 12
    a.fill_kv(12, 3)
    assert a.pos() == 12
    lg = a.step(prompts[:, :1])
    assert np.isfinite(lg).all() and a.pos() == 13
    a.close(); b.close()


@pytest.mark.parametrize("dt", ["q8", "q4"])
def test_host_driver_expert_parallel_matches_one_gpu(tmp_path, dt):
    """moe_generate with the experts sharded over 2 GPUs (moe_ffn_ep in every
    MoE block, 2 of the 4 sequences per rank) greedy-decodes exactly the
    tokens of the one-GPU run of the same model and prompts."""
    import subprocess
    import sys
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("expert parallelism needs one GPU per rank (2 GPUs)")
    exe = os.path.join(os.path.dirname(mh.LIB_PATH), "moe_generate")
    args = ["--layers", "2", "--dtype", dt, "--batch", "4", "--prompt", "6", "--steps", "5", "--seed", "3"]
    one = subprocess.run([exe] + args + ["--out", str(tmp_path / "one")], capture_output=True, text=True,
                         timeout=600)
    assert one.returncode == 0, one.stderr[-2000:]
    ep_dir = tmp_path / "ep"
    ep_dir.mkdir()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    two = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--no-python", "--nnodes=1",
                          "--nproc-per-node=2", "--master-addr", "127.0.0.1",
                          "--master-port", str(29910 + len(dt) + (dt == "q4")), exe] + args +
                         ["--ep-dir", str(ep_dir), "--out", str(tmp_path / "two")],
                         capture_output=True, text=True, timeout=600, env=env)
    assert two.returncode == 0, two.stderr[-3000:]
    want = (tmp_path / "one.0").read_text().split("\n")
    got = (tmp_path / "two.0").read_text().split("\n")[:2] + (tmp_path / "two.1").read_text().split("\n")[:2]
    assert want[:4] == got, (want, got)
    assert '"ep_world": 2' in two.stdout

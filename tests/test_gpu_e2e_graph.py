"""MOE_E2E_GRAPH=1 (graph replay of host-pointer moe_ffn calls) against the
eager path: every call's outputs, top-k and weights bit for bit, across
layers, token counts and rotating host buffers. (The switch stays off by
default: it measured slower than the eager path.)"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def run(tmp_path, graph):
    out = str(tmp_path / f"g{graph}.npz")
    env = dict(os.environ, MOE_E2E_GRAPH=str(graph))
    r = subprocess.run([sys.executable, os.path.join(HERE, "e2e_graph_worker.py"), out], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return np.load(out)


def test_graph_replay_equals_eager(tmp_path):
    eager, graph = run(tmp_path, 0), run(tmp_path, 1)
    assert set(eager.files) == set(graph.files)
    for k in eager.files:
        assert np.array_equal(eager[k], graph[k]), k

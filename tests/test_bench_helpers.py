"""Host-side pieces of bench.py that the driver's numbers rest on: how a strong-scaling workload
deals its streams over the ranks, the algorithmic bytes of a token step behind `step_roofline`,
and the refusal of a `--gpus N` run that was not launched with N ranks."""
import json
import os
import subprocess
import sys

import pytest

import bench
from whisper4j_b200 import ggml

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_strong_scaling_deals_every_stream_once(world):
    cfg = bench.CONFIGS[bench.DEFAULT_CONFIG]
    seen = []
    for rank in range(world):
        ids, total, kind = bench.shard(cfg, rank, world)
        assert kind == "strong" and total == cfg["streams_total"]
        assert len(ids) == total // world  # 256 streams split evenly over 1, 2, 4 or 8 ranks
        assert all(i % world == rank for i in ids)  # stream i -> rank i mod world (whisper4j_b200.shard)
        seen += ids
    assert sorted(seen) == list(range(cfg["streams_total"]))


def test_weak_scaling_gives_every_rank_its_own_streams():
    cfg = bench.CONFIGS["turbo-greedy-32"]
    a, total, kind = bench.shard(cfg, 0, 2)
    b, _, _ = bench.shard(cfg, 1, 2)
    assert kind == "weak" and total == 64 and len(a) == len(b) == 32 and not set(a) & set(b)


def test_step_bytes_of_the_default_workload():
    """Weights (14 d^2 per layer + the embedding, f16) + every stream's cross K/V + every sequence's
    self K/V at the mean context of a 224-token decode after a 4-token prompt."""
    dims = ggml.ARCHS["large-v3-turbo"]
    total, weights = bench.step_bytes(dims, "f16", 256, 1, 224, 4)
    d, L, V = dims.n_text_state, dims.n_text_layer, dims.n_vocab
    assert weights == 14 * d * d * L * 2 + V * d * 2
    cross = 256 * 2 * dims.n_audio_ctx * d * L * 2
    self_kv = 256 * (2 * (4 + 112) * d * L * 2 + 2 * d * L * 2)
    assert total == weights + cross + self_kv == 8794014720


def test_gpus_flag_must_match_the_launched_ranks():
    env = dict(os.environ, WORLD_SIZE="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--gpus", "2"], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 2
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert "WORLD_SIZE" in line["error"]

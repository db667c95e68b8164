"""ShardedEngine (laya_cuda/sharding.py) on the GPU: requests partitioned across engine replicas,
one host thread each, answers returned in request order and equal to a single Engine's within
the probability gate (micro-batches differ, so split-K choices and row packing may differ).
Two replicas on cuda:0 run everywhere; a two-device case runs when two GPUs are present."""
import numpy as np
import pytest

from laya_cuda import Engine
from laya_cuda import synthetic as S
from laya_cuda.sharding import ShardedEngine

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    arch = S.architecture("small", max_len=256)
    return S.write_checkpoint(tmp_path_factory.mktemp("shard"), arch, seed=5), arch


def requests(arch, count=24):
    rng = np.random.default_rng(31)
    return [S.stream_request_texts(rng, arch["vocab"], lengths=(20, 200), questions=(1, 3), options=(2, 9))
            for _ in range(count)]


def close(a, b):
    assert a["usage"] == b["usage"] and list(a["answers"]) == list(b["answers"])
    for key, x in a["answers"].items():
        p = np.array(list(x["probabilities"].values()))
        q = np.array(list(b["answers"][key]["probabilities"].values()))
        assert np.max(np.abs(p - q)) <= 2e-3
        assert abs(x["action"]["act_probability"] - b["answers"][key]["action"]["act_probability"]) <= 2e-3


@pytest.mark.parametrize("devices", [["cuda:0", "cuda:0"], ["cuda:0", "cuda:1"]])
def test_sharded_engine_matches_engine(ckpt, devices):
    if len(set(devices)) > torch.cuda.device_count():
        pytest.skip(f"needs {len(set(devices))} GPUs")
    path, arch = ckpt
    reqs = requests(arch)
    with Engine(path) as engine:
        expected = [engine.predict(state, qs) for state, qs in reqs]
    with ShardedEngine(path, devices=devices, micro_batch=8) as sharded:
        got = sharded.predict_batch(reqs)
        metrics = sharded.last_metrics
    for a, b in zip(got, expected):
        close(a, b)
    assert sum(d["requests"] for d in metrics["devices"]) == len(reqs)
    assert all(d["requests"] > 0 and d["gpu_ms"] > 0 for d in metrics["devices"])
    assert metrics["imbalance"] < 1.2

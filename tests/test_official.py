"""backend="official" (laya_cuda/official.py) on the host: the checkpoint staging and the
CUDA-only guards.  The official SDK is not installed in this image, so a stand-in `laya` module
is injected; nothing here needs a GPU."""
import os
import sys
import types

import pytest

torch = pytest.importorskip("torch")

from laya_cuda import official  # noqa: E402


def test_stage_copies_small_files_and_links_the_weights(tmp_path, monkeypatch):
    src, dst = tmp_path / "ckpt", tmp_path / "staged"
    (src / "tokenizer").mkdir(parents=True)
    (src / "tokenizer" / "tokenizer.json").write_text("{}")
    (src / "rl_agent_config.json").write_text("{}")
    (src / "model.safetensors").write_bytes(b"\0" * 64)
    monkeypatch.setattr(official, "_LINK_BYTES", 32)
    dst.mkdir()
    official._stage(src, dst)
    assert (dst / "tokenizer" / "tokenizer.json").read_text() == "{}"
    # The SDK may rewrite its tokenizer files: those are copies, the large weights a link.
    assert not os.path.samefile(dst / "tokenizer" / "tokenizer.json", src / "tokenizer" / "tokenizer.json")
    assert os.path.samefile(dst / "model.safetensors", src / "model.safetensors")


def test_official_refuses_a_torch_without_cuda(tmp_path, monkeypatch):
    monkeypatch.setitem(sys.modules, "laya", types.ModuleType("laya"))
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="CUDA"):
        official.Official(tmp_path, "cuda:0")


def test_official_refuses_an_agent_on_the_cpu(tmp_path, monkeypatch):
    class Agent:
        def __init__(self, path, device):
            self.device = torch.device("cpu")
            self.model = torch.nn.Linear(2, 2)
    monkeypatch.setitem(sys.modules, "laya", types.SimpleNamespace(Agent=Agent))
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    (tmp_path / "f.json").write_text("{}")
    with pytest.raises(RuntimeError, match="only CUDA runs"):
        official.Official(tmp_path, "cuda:0")


def test_forward_probe_refuses_cpu_inputs():
    model = torch.nn.Linear(2, 2)
    probe = official._CudaProbe(torch, model, torch.device("cuda", 0))
    with pytest.raises(RuntimeError, match="only CUDA runs"):
        model(torch.zeros(1, 2))
    probe.remove()
    model(torch.zeros(1, 2))  # hooks removed

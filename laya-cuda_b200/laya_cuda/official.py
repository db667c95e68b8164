"""backend="official": the unmodified official Laya SDK on a CUDA device.

Kept for API parity with the reference (laya_cuda/official.py:8-72): the SDK runs its own
model on the GPU, timed with CUDA events around its forward pass.  It is a comparison
backend only; the product path is liblaya_b200.so.
"""
import gc
import shutil
import tempfile
from pathlib import Path


class Official:
    def __init__(self, path, device):
        try:
            import torch
            import laya
        except ImportError as error:
            raise ImportError('The official backend needs the "laya" SDK and torch installed') from error
        if not torch.cuda.is_available():
            raise RuntimeError("The official backend requires a CUDA-enabled torch build")
        self.torch = torch
        # The SDK may rewrite tokenizer files; give it a disposable copy of the checkpoint.
        self.temp = tempfile.TemporaryDirectory(prefix="laya-b200-official-")
        target = Path(self.temp.name)
        try:
            for sub in ("tokenizer", "encoder"):
                shutil.copytree(path / sub, target / sub)
            shutil.copy2(path / "rl_agent_config.json", target / "rl_agent_config.json")
            try:
                (target / "model.safetensors").hardlink_to(path / "model.safetensors")
            except OSError:
                shutil.copy2(path / "model.safetensors", target / "model.safetensors")
            self.agent = laya.Agent(str(target), device=device)
            if self.agent.device.type != "cuda":
                raise RuntimeError("Official SDK unexpectedly fell back to CPU")
            self.events = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            stream = lambda: torch.cuda.current_stream(self.agent.device)  # noqa: E731
            self.hooks = [self.agent.model.register_forward_pre_hook(lambda *_: self.events[0].record(stream())),
                          self.agent.model.register_forward_hook(lambda *_: self.events[1].record(stream()))]
            self.gpu_ms = None
        except BaseException:
            self.temp.cleanup()
            raise

    @property
    def precision(self):
        return str(self.agent.dtype)

    def predict(self, state, questions):
        result = self.agent.system_one(state, questions)
        self.torch.cuda.synchronize(self.agent.device)
        self.gpu_ms = self.events[0].elapsed_time(self.events[1])
        return result

    def close(self):
        for hook in self.hooks:
            hook.remove()
        self.agent = None
        gc.collect()
        self.torch.cuda.empty_cache()
        self.temp.cleanup()

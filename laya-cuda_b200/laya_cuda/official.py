"""backend="official": the installed, unmodified Laya SDK as a comparison backend on CUDA.

Engine(backend="official") dispatches here (the reference's engine.py:23-24 does the same).
The SDK owns its model and its whole forward pass; this module only

  * stages the checkpoint where the SDK may edit files (it rewrites its tokenizer settings on
    load): small files are copied into a private directory, the weights file is linked;
  * refuses anything that is not a CUDA run: the SDK's device, every model parameter and
    buffer, and every tensor fed to the model's forward must live on a CUDA device, checked
    at load, at every forward and after every prediction, so a silent CPU fallback can never
    be reported as a GPU number;
  * times the model forward with CUDA events on the SDK's stream (gpu_ms).

It is not the product path: that is liblaya_b200.so behind backend="cuda".
"""
import gc
import os
import shutil
import tempfile
from pathlib import Path

# Files above this size are linked into the staging directory instead of copied.
_LINK_BYTES = 1 << 20


def _stage(checkpoint, into):
    """Mirrors `checkpoint` under `into`: small files copied (the SDK may rewrite them), large
    ones hard-linked when the filesystem allows, copied otherwise."""
    for source in sorted(Path(checkpoint).rglob("*")):
        target = into / source.relative_to(checkpoint)
        if source.is_dir():
            target.mkdir(parents=True, exist_ok=True)
            continue
        target.parent.mkdir(parents=True, exist_ok=True)
        if source.stat().st_size >= _LINK_BYTES:
            try:
                os.link(source, target)
                continue
            except OSError:
                pass
        shutil.copy2(source, target)


class _CudaProbe:
    """Forward hooks on the SDK model: refuse non-CUDA inputs, record the forward's start and
    end events on the model's device stream."""

    def __init__(self, torch, model, device):
        self.torch, self.device = torch, device
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)
        self.input_devices = set()
        self.handles = [model.register_forward_pre_hook(self._enter), model.register_forward_hook(self._leave)]

    def _enter(self, _module, inputs):
        tensors = [x for x in inputs if self.torch.is_tensor(x)]
        where = {x.device.type for x in tensors}
        if not tensors or where != {"cuda"}:
            raise RuntimeError(f"official SDK forward got inputs on {sorted(where) or 'no tensors'}; "
                               "only CUDA runs are compared")
        self.input_devices.update(str(x.device) for x in tensors)
        self.start.record(self.torch.cuda.current_stream(self.device))

    def _leave(self, *_):
        self.end.record(self.torch.cuda.current_stream(self.device))

    def elapsed_ms(self):
        self.torch.cuda.synchronize(self.device)
        return self.start.elapsed_time(self.end)

    def remove(self):
        for handle in self.handles:
            handle.remove()
        self.handles = []


class Official:
    """The SDK agent for one checkpoint on one CUDA device (`predict`, `precision`, `gpu_ms`)."""

    def __init__(self, path, device):
        try:
            import torch
            import laya
        except ImportError as error:
            raise ImportError('backend="official" needs the official "laya" SDK and torch') from error
        if not torch.cuda.is_available():
            raise RuntimeError('backend="official" needs a torch build with CUDA support and a CUDA device')
        self.torch, self.gpu_ms, self.probe = torch, None, None
        self._staging = tempfile.TemporaryDirectory(prefix="laya-b200-sdk-")
        try:
            _stage(Path(path), Path(self._staging.name))
            self.agent = laya.Agent(self._staging.name, device=device)
            self._require_cuda("after loading")
            tensors = [*self.agent.model.parameters(), *self.agent.model.buffers()]
            self.device_info = {"torch_version": torch.__version__, "cuda_build": torch.version.cuda,
                                "gpu": torch.cuda.get_device_name(self.agent.device),
                                "model_devices": sorted({str(t.device) for t in tensors})}
            self.probe = _CudaProbe(torch, self.agent.model, self.agent.device)
        except BaseException:
            self.close()
            raise

    def _require_cuda(self, when):
        if self.agent.device.type != "cuda":
            raise RuntimeError(f"official SDK runs on {self.agent.device} {when}; only CUDA runs are compared")
        tensors = [*self.agent.model.parameters(), *self.agent.model.buffers()]
        if not tensors or any(t.device.type != "cuda" for t in tensors):
            raise RuntimeError(f"official SDK model tensors are not all on CUDA {when}")

    @property
    def precision(self):
        return str(self.agent.dtype)

    def predict(self, state, questions):
        result = self.agent.system_one(state, questions)
        self._require_cuda("after predicting")
        self.device_info["input_devices"] = sorted(self.probe.input_devices)
        self.gpu_ms = self.probe.elapsed_ms()
        return result

    def close(self):
        if self.probe is not None:
            self.probe.remove()
            self.probe = None
        if getattr(self, "agent", None) is not None:
            self.agent = None
            gc.collect()
            self.torch.cuda.empty_cache()
        if self._staging is not None:
            self._staging.cleanup()
            self._staging = None

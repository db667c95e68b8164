"""Model registry: alias -> pinned Hugging Face snapshot or local checkpoint directory.

Same contract as the reference registry (laya_cuda/models.py:1-58): the packaged
models.json is merged with an optional user registry; entries are either {"path": ...}
(resolved relative to the registry file) or {"repo_id": ..., "revision": ...}; a checkpoint
directory must hold the files in FILES.
"""
import json
from pathlib import Path

FILES = ["model.safetensors", "rl_agent_config.json", "encoder/config.json", "tokenizer/*"]
REQUIRED = ("model.safetensors", "rl_agent_config.json", "encoder/config.json", "tokenizer/tokenizer.json")


def read_json(path):
    return json.loads(Path(path).read_text(encoding="utf-8"))


def _valid_entry(alias, entry):
    if not alias.strip() or not isinstance(entry, dict):
        return False
    if set(entry) not in ({"path"}, {"repo_id", "revision"}):
        return False
    return all(isinstance(v, str) and v.strip() for v in entry.values())


def _checkpoints(registry=None):
    """All registry entries, the user's registry overriding the packaged one."""
    sources = [Path(__file__).with_name("models.json")]
    if registry is not None:
        sources.append(Path(registry).expanduser())
    merged = {}
    for source in sources:
        data = read_json(source)
        if not isinstance(data, dict):
            raise ValueError(f"Model registry must be a JSON object: {source}")
        for alias, entry in data.items():
            if not _valid_entry(alias, entry):
                raise ValueError(f"Invalid model entry {alias!r} in {source}; use path or repo_id and revision")
            if "path" in entry:
                entry = {"path": str((source.parent / Path(entry["path"]).expanduser()).resolve())}
            merged[alias] = entry
    return merged


def resolve(model, revision=None, *, registry=None):
    """Checkpoint directory for an alias or a local path; downloads pinned snapshots on demand."""
    path = Path(model).expanduser()
    if not path.is_dir():
        entries = _checkpoints(registry)
        entry = entries.get(str(model))
        if entry is None:
            raise FileNotFoundError(f"Unknown alias or missing local checkpoint: {model}")
        if "path" in entry:
            path = Path(entry["path"])
        else:
            from huggingface_hub import snapshot_download
            path = Path(snapshot_download(entry["repo_id"], revision=revision or entry["revision"],
                                          allow_patterns=FILES))
    for name in REQUIRED:
        if not (path / name).is_file():
            raise FileNotFoundError(f"Incomplete checkpoint: {path / name}")
    return path.resolve()


def adapter(path):
    """The model adapter for a checkpoint directory (Laya checkpoints carry rl_agent_config.json)."""
    if not (path / "rl_agent_config.json").is_file():
        raise ValueError("No compatible model adapter")
    from .laya import Laya
    return Laya(path)

"""Runtime and build metadata reported by ``/health`` and result JSON (reference fp/runtime_metadata.py)."""

from __future__ import annotations

import torch

from .. import __version__


def package_version() -> str:
    return __version__


def runtime_info(device: torch.device | None = None) -> dict[str, object]:
    info: dict[str, object] = {"package": "0709_b200", "version": __version__, "torch": torch.__version__,
                               "cuda_runtime": torch.version.cuda}
    if device is not None and device.type == "cuda" and torch.cuda.is_available():
        props = torch.cuda.get_device_properties(device)
        info.update({"gpu": props.name, "sm": f"{props.major}.{props.minor}", "sms": props.multi_processor_count,
                     "hbm_gb": round(props.total_memory / 2 ** 30, 1)})
    return info

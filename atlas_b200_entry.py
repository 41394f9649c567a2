"""Console-script targets of the installed package.

The package folder ``0709_b200`` starts with a digit, which entry-point references may not name
directly; each function here imports the command's module and runs its ``main``.
"""

from __future__ import annotations

import importlib


def _run(module: str) -> int:
    return int(importlib.import_module(f"0709_b200.{module}").main() or 0)


def clean_run() -> int:
    return _run("serving.cli")


def target_server() -> int:
    return _run("serving.target_server")


def edge() -> int:
    return _run("serving.distributed_system")


def check_equivalence() -> int:
    return _run("serving.check_equivalence")


def diagnostics() -> int:
    return _run("serving.diagnostics")


def eval_gsm8k() -> int:
    return _run("eval.gsm8k")


def eval_mtbench() -> int:
    return _run("eval.mtbench")


def eval_sweep() -> int:
    return _run("eval.sweep")


def compare_interventions() -> int:
    return _run("eval.compare_interventions")

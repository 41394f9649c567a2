"""atlas-b200: asynchronous tree/forest speculative decoding, built for B200 (sm_100a).

Import the package with ``importlib.import_module("0709_b200")`` (the folder
name starts with a digit); command-line tools run as ``python -m 0709_b200.<tool>``.

Layout:
- ``models``   Llama configs, seeded random-init weights, fp32 oracle;
- ``ops``      native extensions (C++ page pool, sm_100a kernels) and PyTorch op semantics;
- ``runtime``  route store, frontier/builders, drafter and target runtimes, engine;
- ``serving``  async/serial coordinators, RPC (HTTP + in-process), CLIs, sessions;
- ``parallel`` tensor parallelism and its fused peer-memory collectives;
- ``utils``    timeline, interventions, timing and clocks.
"""

__version__ = "0.1.0"

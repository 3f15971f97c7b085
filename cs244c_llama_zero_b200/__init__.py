"""B200-native ZeRO research harness for LLaMA-style training.

Subpackages:

* ``models``   - LLaMA model (eager PyTorch oracle backend and sm_100a kernel backend)
* ``ops``      - hand-written CUDA kernels for sm_100a and their autograd wrappers
* ``parallel`` - collectives (ring / NCCL / NVLink symmetric-memory kernels) and ZeRO 0-3 engines
* ``profiler`` - timers, memory tracker, FLOP accounting, overlap efficiency
* ``data``     - synthetic, uniform-random and FineWeb token streams
* ``train``    - the training session API used by the CLIs and the benchmark
* ``experiments`` / ``analysis`` - experiment harness, tuning workflows and reports
"""

__version__ = "0.1.0"

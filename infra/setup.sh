#!/usr/bin/env bash
# Build the sm_100a extension in place and check that the package imports.
set -euo pipefail
here="$(cd "$(dirname "$0")/.." && pwd)"
cd "$here"
if [[ -f requirements.txt ]]; then python -m pip install -r requirements.txt || true; fi
TORCH_CUDA_ARCH_LIST=10.0a MAX_JOBS="${MAX_JOBS:-8}" python setup.py build_ext --inplace
python -c "import cs244c_llama_zero_b200, torch; from cs244c_llama_zero_b200 import ops; print('extension:', ops.extension_available(), 'cuda:', torch.cuda.is_available())"

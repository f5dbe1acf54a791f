#!/usr/bin/env bash
# Run a test suite written for the reference package (``import torch_einshard``)
# against this framework through the compat import name, on 1 process and on
# N gloo ranks (the reference runs its suite under torchrun with 8 processes).
#
#   compat/run_reference_suite.sh <tests-dir> [nproc]
set -euo pipefail
TESTS=${1:?usage: run_reference_suite.sh <tests-dir> [nproc]}
NPROC=${2:-8}
HERE=$(cd "$(dirname "$0")" && pwd)
ROOT=$(cd "$HERE/.." && pwd)
export PYTHONPATH="$HERE:$ROOT${PYTHONPATH:+:$PYTHONPATH}"
python -m pytest "$TESTS" -q -p no:cacheprovider
python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NPROC" --master-addr 127.0.0.1 \
    --master-port "${MASTER_PORT:-29790}" -m pytest "$TESTS" -q -p no:cacheprovider

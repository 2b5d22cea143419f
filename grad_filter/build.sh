#!/usr/bin/env bash
# Onboarding step 2: regenerate the node handlers and rebuild the native extensions in-tree.
set -euo pipefail
cd "$(dirname "$0")/.."
python -m centrifuge_b200.filter.codegen
python setup.py build_ext --inplace

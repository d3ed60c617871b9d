#!/usr/bin/env bash
# Install the UNMODIFIED reference (wwillchen/ebr) into baseline/_ref with the offline pip command of the benchmark
# contract. The reference ships no packaging metadata: its pyproject.toml holds only a ruff section, and setuptools'
# flat-layout discovery refuses a tree with four top-level packages (models, utils, dataset, evaluators). So the tree is
# copied to a scratch directory, a setup.py naming those packages is added to the COPY (no reference file is edited),
# and pip installs the copy. The result under baseline/_ref is the reference's own source files, byte for byte.
#
#   baseline/install_reference.sh /path/to/reference/tree
set -euo pipefail
SRC="${1:?usage: install_reference.sh <reference tree>}"
HERE="$(cd "$(dirname "$0")" && pwd)"
TMP="$(mktemp -d /tmp/ebr_ref_pkg.XXXXXX)"
cp -r "$SRC"/. "$TMP"/
cat > "$TMP/setup.py" <<'PY'
from setuptools import setup

setup(
    name="ebr-reference",
    version="0.0.0",
    packages=["models", "models.fused_attn", "utils", "dataset", "evaluators"],
    package_data={"dataset": ["*.npz"]},
)
PY
rm -rf "$HERE/_ref"
python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse --target "$HERE/_ref" "$TMP"
rm -rf "$TMP"
# The installed modules must equal the reference's files.
for f in models/attention.py models/energy.py models/layers.py models/sxm.py models/fused_attn/ops.py \
         models/fused_attn/triton_kernels.py models/fused_attn/reference.py models/fused_attn/rope_split.py; do
  cmp "$SRC/$f" "$HERE/_ref/$f"
done
echo "installed the reference into $HERE/_ref"

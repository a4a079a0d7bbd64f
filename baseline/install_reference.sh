#!/usr/bin/env bash
# Install the reference package (nmquan1503/selective-attention, pure Python + Triton)
# into baseline/_ref, offline and without its dependencies (torch and packaging are
# already in the image). The build writes egg-info next to its sources, so it runs on a
# temporary copy of the (read-only) checkout.
#
#   baseline/install_reference.sh [REFERENCE_CHECKOUT]
#
# REFERENCE_CHECKOUT defaults to $SA_REFERENCE_ROOT. baseline/_ref is git-ignored; the
# tests that run the reference's SSM layer through shim.install() import it from there.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
src="${1:-${SA_REFERENCE_ROOT:-}}"
if [ -z "$src" ] || [ ! -f "$src/pyproject.toml" ]; then
  echo "usage: $0 REFERENCE_CHECKOUT (a directory holding the reference's pyproject.toml)" >&2
  exit 2
fi
tmp="$(mktemp -d)"
trap 'rm -rf "$tmp"' EXIT
cp -r "$src" "$tmp/src"
python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse --no-deps \
  --target "$here/_ref" --upgrade "$tmp/src"

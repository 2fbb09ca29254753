#!/usr/bin/env bash
# Builds the serving image from the repository root (deploy/Dockerfile).
#   deploy/build_image.sh [tag] [extra docker build args...]
set -euo pipefail
cd "$(dirname "$0")/.."
tag="${1:-k8v4-b200:latest}"
shift || true
docker build -f deploy/Dockerfile -t "$tag" "$@" .
echo "built $tag; run: docker run --gpus all --ipc=host -p 8000:8000 $tag --help"

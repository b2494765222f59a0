#!/bin/bash
# Show what cgroup v2 limits do to a training process: run the reader inside
# a container with a memory cap, no swap and 1.5 CPUs.
#
#   bash deploy/cgroups_demo.sh [image]
set -euo pipefail
IMAGE=${1:-python:3.12-slim}
docker run --rm --memory=512m --memory-swap=512m --cpus=1.5 \
  -v "$PWD":/w -w /w "$IMAGE" \
  python -c "import runpy, sys; sys.path.insert(0, '/w'); runpy.run_module('gpt2_harness_b200.cluster.cgroups', run_name='__main__')"

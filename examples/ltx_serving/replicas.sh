#!/usr/bin/env bash
# Launch REPLICAS x CP-GPU replicas of serve.py on one node, all sharing ONE host copy of the
# streamed weights (--shm-namespace), behind nginx on :8080.
#   PROFILE_DIR=/tmp/ltx_profile REPLICAS=8 CP=1 examples/ltx_serving/replicas.sh
# (profile first: python examples/ltx_serving/serve.py profile --profile-dir "$PROFILE_DIR")
# NUMA_INTERLEAVE=1 spreads the shared weight pages over every memory node: the SHM creator
# interleaves each weight segment before writing it (FT_SHM_NUMA_INTERLEAVE=1), and every
# replica runs under an interleave process policy. A host that refuses the policy stops the
# launch before any worker starts. Use a fresh SHM namespace when changing it: existing pages
# keep their node.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
PROFILE_DIR="${PROFILE_DIR:?set PROFILE_DIR to the saved profiles}"
REPLICAS="${REPLICAS:-8}"
CP="${CP:-1}"
NS="${SHM_NAMESPACE:-ltx_$(id -u)}"
PREFIX=()
if [ "${NUMA_INTERLEAVE:-0}" = "1" ]; then
  python -m flextensor_b200.shm.numa probe >/dev/null || {
    echo "NUMA_INTERLEAVE=1: the host refused an interleave policy (containers need SYS_NICE)" >&2
    exit 1
  }
  export FT_SHM_NUMA_INTERLEAVE=1
  PREFIX=(python -m flextensor_b200.shm.numa exec --)
fi
pids=()
for ((r = 0; r < REPLICAS; r++)); do
  first=$((r * CP))
  gpus=$(seq -s, "$first" $((first + CP - 1)))
  port=$((8000 + r))
  if [ "$CP" -gt 1 ]; then
    CUDA_VISIBLE_DEVICES="$gpus" "${PREFIX[@]}" python -m torch.distributed.run --nnodes=1 --nproc-per-node "$CP" \
      --master-addr 127.0.0.1 --master-port $((29500 + r)) "$HERE/serve.py" serve \
      --profile-dir "$PROFILE_DIR" --port "$port" --shm-namespace "$NS" &
  else
    CUDA_VISIBLE_DEVICES="$gpus" "${PREFIX[@]}" python "$HERE/serve.py" serve --profile-dir "$PROFILE_DIR" --port "$port" \
      --shm-namespace "$NS" &
  fi
  pids+=($!)
done
trap 'kill "${pids[@]}" 2>/dev/null || true' EXIT INT TERM
nginx -c "$HERE/nginx.conf" -g "daemon off;"

#!/usr/bin/env bash
# Launch REPLICAS x CP-GPU replicas of serve.py on one node, all sharing ONE host copy of the
# streamed weights (--shm-namespace), behind nginx on :8080.
#   PROFILE_DIR=/tmp/ltx_profile REPLICAS=8 CP=1 examples/ltx_serving/replicas.sh
# (profile first: python examples/ltx_serving/serve.py profile --profile-dir "$PROFILE_DIR")
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
PROFILE_DIR="${PROFILE_DIR:?set PROFILE_DIR to the saved profiles}"
REPLICAS="${REPLICAS:-8}"
CP="${CP:-1}"
NS="${SHM_NAMESPACE:-ltx_$(id -u)}"
pids=()
for ((r = 0; r < REPLICAS; r++)); do
  first=$((r * CP))
  gpus=$(seq -s, "$first" $((first + CP - 1)))
  port=$((8000 + r))
  if [ "$CP" -gt 1 ]; then
    CUDA_VISIBLE_DEVICES="$gpus" python -m torch.distributed.run --nnodes=1 --nproc-per-node "$CP" \
      --master-addr 127.0.0.1 --master-port $((29500 + r)) "$HERE/serve.py" serve \
      --profile-dir "$PROFILE_DIR" --port "$port" --shm-namespace "$NS" &
  else
    CUDA_VISIBLE_DEVICES="$gpus" python "$HERE/serve.py" serve --profile-dir "$PROFILE_DIR" --port "$port" \
      --shm-namespace "$NS" &
  fi
  pids+=($!)
done
trap 'kill "${pids[@]}" 2>/dev/null || true' EXIT INT TERM
nginx -c "$HERE/nginx.conf" -g "daemon off;"

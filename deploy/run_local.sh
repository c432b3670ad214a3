#!/usr/bin/env bash
# Start the whole stack locally in the foreground (Ctrl-C stops everything):
# control plane, the kv-pool byte service, node storage services (agent + transfer +
# kv byte store), one worker and the HTTP router. Run from the repository root:
#   ./deploy/run_local.sh            # LAKE_MODEL_BACKEND=mock -> tiny CPU model
#   LAKE_MODEL_BACKEND=llama3-8b LAKE_DEVICE=cuda ./deploy/run_local.sh
#   LAKE_PD_PAIR=1 ./deploy/run_local.sh   # the worker as a PD-split pair (prefill + decode process)
#   LAKE_WORKERS=2 ./deploy/run_local.sh   # a second worker (worker-1 on LAKE_WORKER1_ADDR)
#   ./deploy/smoke.sh                # in another shell (LAKE_WORKERS=2: ./deploy/smoke_pool.sh)
# Every worker's storage agent is the remote pool agent (LAKE_CP_ADDR + LAKE_KV_ADDR): finished
# requests' KV pages are written back to the kv-pool and any worker pulls pool-held prefixes.
set -euo pipefail
ROOT="$(cd "$(dirname "$0")/.." && pwd)"
cd "$ROOT"

export LAKE_CP_ADDR="${LAKE_CP_ADDR:-127.0.0.1:50051}"
export LAKE_KV_ADDR="${LAKE_KV_ADDR:-127.0.0.1:50052}"
export LAKE_WORKER_BIND="${LAKE_WORKER_BIND:-127.0.0.1:50053}"
export LAKE_WORKER_ADDR="${LAKE_WORKER_ADDR:-127.0.0.1:50053}"
export LAKE_AGENT_ADDR="${LAKE_AGENT_ADDR:-127.0.0.1:50054}"
export LAKE_HTTP_ADDR="${LAKE_HTTP_ADDR:-127.0.0.1:8080}"
export LAKE_MODEL_BACKEND="${LAKE_MODEL_BACKEND:-mock}"
export LAKE_SERVED_MODEL_NAME="${LAKE_SERVED_MODEL_NAME:-mock-llm}"
export LAKE_NODE_ID="${LAKE_NODE_ID:-worker-0}"
export LAKE_WORKER1_ADDR="${LAKE_WORKER1_ADDR:-127.0.0.1:50055}"
if [[ "${LAKE_WORKERS:-1}" == "2" ]]; then
  export LAKE_WORKER_NODES="worker-0=$LAKE_WORKER_ADDR,worker-1=$LAKE_WORKER1_ADDR"
fi
PY="${PYTHON:-python}"

wait_tcp() {
  local hostport="$1" name="$2" tries="${3:-240}"
  local host="${hostport%:*}" port="${hostport##*:}"
  for ((i=1; i<=tries; i++)); do
    if (echo >/dev/tcp/"$host"/"$port") >/dev/null 2>&1; then
      echo "  ready: $name ($hostport)"
      return 0
    fi
    sleep 0.25
  done
  echo "ERROR: timeout waiting for $name ($hostport)" >&2
  return 1
}

PIDS=()
cleanup() {
  for p in "${PIDS[@]:-}"; do kill "$p" 2>/dev/null || true; done
}
trap cleanup EXIT INT TERM

for hp in "$LAKE_CP_ADDR" "$LAKE_KV_ADDR" "$LAKE_WORKER_ADDR" "$LAKE_WORKER1_ADDR" "$LAKE_AGENT_ADDR" "$LAKE_HTTP_ADDR"; do
  if (echo >/dev/tcp/"${hp%:*}"/"${hp##*:}") >/dev/null 2>&1; then
    echo "ERROR: $hp already in use; stop the old stack first" >&2
    exit 1
  fi
done

"$PY" -c "import lake_b200._host" 2>/dev/null || "$PY" -m lake_b200._build

echo "==> control plane"
"$PY" -m lake_b200.services.controlplane & PIDS+=($!)
wait_tcp "$LAKE_CP_ADDR" controlplane
echo "==> kv-pool"
"$PY" -m lake_b200.services.kvpool & PIDS+=($!)
wait_tcp "$LAKE_KV_ADDR" kv-pool
echo "==> node services"
"$PY" -m lake_b200.services.node & PIDS+=($!)
wait_tcp "$LAKE_AGENT_ADDR" node-services
if [[ "${LAKE_PD_PAIR:-0}" == "1" ]]; then
  echo "==> PD worker pair ($LAKE_MODEL_BACKEND)"
  "$PY" -m lake_b200.runtime.pd_pair --bind "$LAKE_WORKER_BIND" & PIDS+=($!)
else
  echo "==> worker ($LAKE_MODEL_BACKEND)"
  "$PY" -m lake_b200.runtime & PIDS+=($!)
fi
wait_tcp "$LAKE_WORKER_ADDR" worker 1200
if [[ "${LAKE_WORKERS:-1}" == "2" ]]; then
  echo "==> second worker ($LAKE_MODEL_BACKEND)"
  LAKE_NODE_ID=worker-1 LAKE_WORKER_BIND="$LAKE_WORKER1_ADDR" "$PY" -m lake_b200.runtime & PIDS+=($!)
  wait_tcp "$LAKE_WORKER1_ADDR" worker-1 1200
fi
echo "==> router"
"$PY" -m lake_b200.router & PIDS+=($!)
wait_tcp "$LAKE_HTTP_ADDR" router
echo "stack up: http://$LAKE_HTTP_ADDR/v1/chat/completions"
wait

#!/usr/bin/env bash
# Two chat requests sharing a 48-character system prefix (3 full 16-token
# blocks under the mock tokenizer): the first is cold, the second must reuse
# at least 3 blocks. Needs ./deploy/run_local.sh running.
set -euo pipefail
BASE="${LAKE_SMOKE_BASE:-http://127.0.0.1:8080}"
URL="$BASE/v1/chat/completions"
SYS='AAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAAA'

for ((i=1; i<=120; i++)); do
  if curl -sf "$BASE/healthz" >/dev/null; then break; fi
  if [[ $i -eq 120 ]]; then echo "ERROR: router not ready"; exit 1; fi
  sleep 0.25
done

post() {
  curl -sS "$URL" -H 'Content-Type: application/json' \
    -d "{\"model\":\"mock-llm\",\"messages\":[{\"role\":\"system\",\"content\":\"$SYS\"},{\"role\":\"user\",\"content\":\"$1\"}],\"max_tokens\":4}"
}
field() { python3 -c "import sys,json; print(json.load(sys.stdin)['lake']['$1'])"; }

A="$(post hello-AAA)"; echo "$A"
sleep 0.5  # let the router's view mirror catch the worker's block registration
B="$(post hello-BBB)"; echo "$B"
RA="$(echo "$A" | field reused_blocks)"; RB="$(echo "$B" | field reused_blocks)"
echo "Req A reused=$RA mode=$(echo "$A" | field mode); Req B reused=$RB mode=$(echo "$B" | field mode)"
[[ "$RA" -eq 0 ]] || { echo "FAIL: Req A should be cold"; exit 1; }
[[ "$RB" -ge 3 ]] || { echo "FAIL: Req B should reuse >= 3 blocks"; exit 1; }
echo "PASS"

#!/usr/bin/env bash
# KV reuse through the pool between two workers (needs LAKE_WORKERS=2 ./deploy/run_local.sh):
# worker-0 serves a prompt and writes its KV pages back to the kv-pool; worker-1, which never
# saw it, serves the same prompt plus a suffix and must reuse the prompt's full blocks, pulled
# from the pool at admission (reused_blocks >= 3 while its own prefix cache was cold).
set -euo pipefail
W0="${LAKE_WORKER_ADDR:-127.0.0.1:50053}"
W1="${LAKE_WORKER1_ADDR:-127.0.0.1:50055}"
MODEL="${LAKE_SERVED_MODEL_NAME:-mock-llm}"
PY="${PYTHON:-python}"
exec "$PY" - "$W0" "$W1" "$MODEL" <<'PYEOF'
import sys

import grpc

from lake_b200.api import proto

w0, w1, model = sys.argv[1:4]
pb = proto.messages()
prompt = [(7 * i + 3) % 1000 + 1 for i in range(60)]  # 3 full 16-token blocks + 12 tokens


def gen(addr, rid, toks):
    stub = proto.Stub(grpc.insecure_channel(addr), "WorkerService")
    return stub.Generate(pb.GenerateRequest(request_id=rid, model_id=model, prompt_tokens=toks, max_new_tokens=4,
                                            exec_mode="COLOCATED"), timeout=120)


a = gen(w0, "smoke-pool-a", prompt)
b = gen(w1, "smoke-pool-b", prompt + [11, 12, 13])
print(f"worker-0 reused={a.reused_blocks} tokens={list(a.output_tokens)}")
print(f"worker-1 reused={b.reused_blocks} tokens={list(b.output_tokens)}")
if a.reused_blocks != 0:
    sys.exit("FAIL: worker-0 should be cold")
if b.reused_blocks < 3:
    sys.exit("FAIL: worker-1 should reuse >= 3 blocks pulled from the pool")
print("PASS")
PYEOF

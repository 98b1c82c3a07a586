"""One rank of the multi-process bench test (launched by torchrun with
JL_DIST_BACKEND=gloo): exercises bench.Dist and bench.aggregate on host cores."""
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

dist = bench.Dist()
r = dist.rank
dist.barrier()
# rank r generated 64 + r tokens in 100 * (r + 1) ms of device time and 1 + r s of wall time
value, e2e, tokens, slowest_ms = bench.aggregate(dist, 64 + r, 100.0 * (r + 1), 1.0 + r)
dist.barrier()
out = Path(os.environ["JL_DIST_OUT"]) / f"rank{r}.json"
out.write_text(json.dumps({"rank": r, "world": dist.world, "value": value, "e2e": e2e, "tokens": tokens, "slowest_ms": slowest_ms}))
dist.close()

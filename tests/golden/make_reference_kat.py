"""Regenerates reference_kat.json from the reference repository's own published
forward losses (run where the reference checkout is available; the JSON is the
committed fixture the tests read).

Every entry is a forward+loss of the reference engine with its own init
(ModelWeights::random, crates/engine/src/full_model.rs:132-141 and
LayerWeights::random, crates/engine/src/layer.rs:1509-1524) on the benchmark
tokens (i*31+7) % 8192 with targets shifted by one
(crates/engine/tests/bench_fwd_only_scale.rs:110-115), seq 512, softcap 0.
Because that init zeroes Wo and W2, every layer is an exact identity and the
loss depends only on (dim, vocab, seq): embedding, final RMSNorm, tied head, CE.

Sources:
  results/forward_utilization/scale_ladder.json  -- `loss` of each ladder entry
  README.md "600m-A ... Forward pass... loss=9.0108" (4 decimals)

usage: python tests/golden/make_reference_kat.py /path/to/reference
"""
import json
import re
import sys
from pathlib import Path


def main(ref: Path) -> None:
    out = []
    ladder = json.loads((ref / "results/forward_utilization/scale_ladder.json").read_text())
    for e in ladder:
        out.append(dict(name=e["name"], dim=e["dim"], hidden=e["hidden"], heads=e["heads"],
                        nlayers=e["nlayers"], seq=e["seq"], vocab=8192, loss=e["loss"],
                        decimals=6, source="results/forward_utilization/scale_ladder.json"))
    readme = (ref / "README.md").read_text()
    m = re.search(r"600m-A.*?1536d/4096h/20L/seq512.*?loss=([0-9.]+)", readme, re.S)
    if m:
        out.insert(0, dict(name="600m-A", dim=1536, hidden=4096, heads=12, nlayers=20, seq=512,
                           vocab=8192, loss=float(m.group(1)), decimals=4, source="README.md"))
    path = Path(__file__).with_name("reference_kat.json")
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {len(out)} entries to {path}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(Path(sys.argv[1]))

"""Writes tests/golden/precision_map_factorized.json: the reference's example
FactorizedPrior precision map (examples/precision_configs/FactorizedPrior/
kodak-20261026T091208.288386Z.json of the reference), schema 4, with its probe
records, recovery steps and P_ch sweep measurements dropped to keep the
fixture small.  Every field the loader checks is kept; the tests rewrite the
model fingerprint and P_ch for their own models.

    python tests/golden/make_precision_fixture.py <reference checkout>
"""

import json
import sys
from pathlib import Path

src = Path(sys.argv[1]) / "examples/precision_configs/FactorizedPrior/kodak-20261026T091208.288386Z.json"
data = json.loads(src.read_text())
data["probe_records"] = []
data["recovery_steps"] = []
data["records_path"] = None
data["recovery_path"] = None
if data.get("p_ch_selection"):
    data["p_ch_selection"] = {k: v for k, v in data["p_ch_selection"].items() if k != "measurements"}
out = Path(__file__).with_name("precision_map_factorized.json")
out.write_text(json.dumps(data, sort_keys=True, indent=1) + "\n")
print(out, out.stat().st_size)

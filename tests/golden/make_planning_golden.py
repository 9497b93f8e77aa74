"""Golden outputs of the reference's planning helpers (dl1683/matrix-numbers code/digit_gemm.py: coprime_ip
:1224-1241, int8_crt :1244-1249, cmd_chain :1252-1291), produced by importing the reference module in the build
container (it needs numpy and scipy only; cmd_chain's file output is captured instead of written).

    python tests/golden/make_planning_golden.py /path/to/reference    # writes tests/golden/planning_golden.json
"""
import json
import math
import os
import sys

CASES_INT8 = [(53, 1024), (53, 4096), (53, 16384), (53, 262144), (8, 4096), (16, 4096), (24, 1024), (31, 65536)]
CASES_IP = [([(m, 1) for m in range(2, 257)], 100.0), ([(m, (m % 7) + 1) for m in range(100, 257)], 64.0),
            ([(m, 3) for m in (243, 245, 247, 249, 251, 253, 255, 256)], 40.0)]


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "code"))
    import digit_gemm as dg
    out = {"int8_crt": [], "coprime_ip": [], "chain": None}
    for b, k in CASES_INT8:
        mods, n = dg.int8_crt(b, k)
        out["int8_crt"].append({"b": b, "k": k, "mods": mods, "n": n})
    for cands, target in CASES_IP:
        mods, cost = dg.coprime_ip(cands, target)
        out["coprime_ip"].append({"cands": cands, "target": target, "mods": mods, "cost": cost})
    cap = {}
    dg._save = lambda name, obj: cap.__setitem__(name, obj)
    dg.cmd_chain()
    out["chain"] = cap["chain_cost_model.json"]
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "planning_golden.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=0)
    print("wrote", path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_ROOT", "reference"))

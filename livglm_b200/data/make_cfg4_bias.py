"""Fit and store the config-4 Zipf(1.2) correction bias.

    python -m livglm_b200.data.make_cfg4_bias

Writes livglm_b200/data/cfg4_zipf_bias.json (see livglm_b200/workloads.py for
the fit); deterministic, runs on the CPU in a few seconds.
"""

from __future__ import annotations

import json

from livglm_b200.workloads import CFG4_BIAS_PATH, calibrate_zipf_bias


def main() -> None:
    res = calibrate_zipf_bias()
    CFG4_BIAS_PATH.write_text(json.dumps(res, indent=1) + "\n")
    st = res["stats"]
    print(f"beta={res['beta']:.4f} l1={res['l1_to_target']:.3f} max/mean={st['max_over_mean']:.2f} "
          f"experts used={st['experts_used']}")


if __name__ == "__main__":
    main()

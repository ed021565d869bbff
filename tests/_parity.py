"""Action parity of the policy steps against the reference's committed fixtures.

Every policy test compares its actions with the reference's through
check_actions(label, got, want, tol): configurations listed in BIT_IDENTICAL
must equal the reference bit for bit (they do on the B200 today, so any
regression shows); the others must stay within `tol` (the north star's
action-chunk max-abs 1e-3 unless a test says otherwise). VLA_PARITY_LOG=<file>
appends one JSON line per check (label, max-abs, bits equal) for the record.
"""
import json
import os

import numpy as np

# every configuration the policy tests check, bit-identical on the B200
BIT_IDENTICAL = {
    "act-small-m63",
    "act-small-m0",
    "act-small-m31",
    "act-small-m40",
    "act-base-m63",
    "dp-small-m3",
    "dp-small-m0",
    "dp-small-m1",
    "dp-small-m3-ddpm",
    "dp-small-m3-nonoise",
    "dp-base-m3",
    "dp-base-m0",
    "dp-edge-m3",
    "dp-edge-m0",
    "dp-edge-m2",
    "dp-deep-m3",
    "dp-deep-m0",
    "octo-small-m63",
    "octo-small-m0",
    "octo-small-m31",
    "octo-erf-m63",
    "octo-small-m63-readout",
    "octo-small-m63-nowrist",
    "octo-small-m63-pad",
    "octo-small-m63-w1",
    "octo-small-m63-seed",
    "octo-base-m63",
    "smolvla-small-m63-plain",
    "smolvla-small-m0-plain",
    "smolvla-small-m59-plain",
    "smolvla-small-m63-rtc",
    "smolvla-small-m63-seed",
    "smolvla-edge-m63",
    "smolvla-edge-m0",
    "smolvla-base-m63",
}


def check_actions(label, got, want, tol):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{label}: shape {got.shape} != {want.shape}"
    err = float(np.abs(got.astype(np.float64) - want.astype(np.float64)).max()) if want.size else 0.0
    same = bool(np.array_equal(got, want))
    print(f"{label}: max-abs vs reference {err:.3g}{' (bit-identical)' if same else ''}")
    log = os.environ.get("VLA_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(json.dumps({"label": label, "max_abs": err, "bit_identical": same}) + "\n")
    if label in BIT_IDENTICAL:
        assert same, f"{label}: no longer bit-identical to the reference (max-abs {err:.3g})"
    else:
        assert err <= tol, f"{label}: max-abs {err:.3g} above {tol}"

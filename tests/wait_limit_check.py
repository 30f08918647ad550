"""Run in a child process by test_gpu_wait_limit.py: drives the conv kernel's
bounded waits to their limit and checks that the context stays usable.

1. The wait limit is set to 20 ms (sc_set_wait_limit_ns).
2. With SC_TC_TEST_STALL=1 the single-CTA kernel's MMA warp waits on a barrier
   that nothing completes; the producers fill the stage ring and then wait for
   free stages, the epilogue waits for an accumulator: every role reaches the
   limit, raises FAULT_WAIT_TIMEOUT and drains (no address of this mode comes
   from uninitialised memory: the producers gather rows of a valid map).
3. The fault word reads FAULT_WAIT_TIMEOUT, and a normal conv afterwards, with
   the default limit, matches the oracle.
Prints one JSON line; exit code 0 when every check passes."""
import json
import os
import sys
import time

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import oracle  # noqa: E402
from bevy_synth_b200 import _lib, synth  # noqa: E402
from bevy_synth_b200 import flex_gmm as F  # noqa: E402


def main():
    dev = torch.device("cuda:0")
    coords = synth.morton_sort(synth.unique_cells(0, synth.sphere_shell(24, (12.0, 12.0, 12.0), 8.0, 1.0)))
    c = 128
    rng = np.random.default_rng(2)
    x = rng.standard_normal((coords.shape[0], c)).astype(np.float32)
    w = (0.05 * rng.standard_normal((c, 3, 3, 3, c))).astype(np.float32)
    b = np.zeros(c, np.float32)
    cfg = F.SparseSubmConvConfig.subm3(c, c)
    ct = torch.as_tensor(coords, device=dev)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, ct)
    xt = torch.as_tensor(x, device=dev).to(torch.bfloat16)
    wt = torch.as_tensor(w, device=dev).to(torch.bfloat16)
    bt = torch.as_tensor(b, device=dev)
    out = {"tensor_cores": F.uses_tensor_cores(cfg, torch.bfloat16), "rows": int(coords.shape[0])}
    assert _lib.device_fault() == 0
    _lib.set_wait_limit_ns(20_000_000)
    os.environ["SC_TC_TEST_STALL"] = "1"
    t0 = time.time()
    F.sparse_subm_conv_forward(cfg, xt, nbr, wt, bt)
    torch.cuda.synchronize()
    out["stalled_launch_s"] = round(time.time() - t0, 3)
    del os.environ["SC_TC_TEST_STALL"]
    out["fault"] = _lib.device_fault()
    _lib.set_wait_limit_ns(0)
    y = F.sparse_subm_conv_forward(cfg, xt, nbr, wt, bt).float().cpu().numpy()
    ref = oracle.bf16_round(oracle.subm_conv_flex(oracle.OracleConfig(c, c), oracle.bf16_round(w), b,
                                                  oracle.bf16_round(x), nbr.cpu().numpy(), threads=8))
    out["rel_after"] = float(np.linalg.norm(y - ref) / np.linalg.norm(ref))
    out["fault_after"] = _lib.device_fault()
    out["ok"] = bool(out["tensor_cores"] and out["fault"] & _lib.FAULT_WAIT_TIMEOUT and out["rel_after"] <= 1e-2
                     and out["fault_after"] == 0)
    print(json.dumps(out), flush=True)
    sys.exit(0 if out["ok"] else 1)


if __name__ == "__main__":
    main()

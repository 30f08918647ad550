"""Writes the golden fixtures under tests/golden/.

Sources (paths in the mosure/bevy_synth repository):
* kat_neighbor_voxels.json: burn_trellis/src/runtime_model/sparse_decoder_tests.rs:189-236
  (coords x=0,1; input [1,2]; 3x1x1 weights [10,1,100]; expected [201, 12]).
* kat_halo_chunk.json: sparse_decoder_tests.rs:238-292 (full map row 0
  [-1,0,1]; map rebuilt from the one-row chunk [-1,0,-1]).
* lcg_seed42.json: the reference LCG (burn_flex_gmm/src/lib.rs:764-778)
  evaluated here with exact integer arithmetic and IEEE-single rounding done
  through ``struct`` -- a formulation independent of oracle.Lcg.
* dup_coords.json: the duplicate-coordinate case of
  burn_flex_gmm/src/wgpu/tests.rs:1801-1853 (line of 128 + rows 17,32,17,32
  appended, 3x3x1 kernel); its expected map is the lowest-row rule computed
  by a brute-force scan in this script (the reference's own Scan builder,
  neighbor_kernels.rs:3-46).

Run:  python tests/golden/make_golden.py
"""
import json
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))


def f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", x))[0]


def lcg_values(seed: int, n: int):
    state = (seed | 1) & (2**64 - 1)
    out = []
    umax = f32(float(2**32 - 1))
    for _ in range(n):
        state = (state * 6364136223846793005 + 1) & (2**64 - 1)
        bits = ((state >> 40) & 0xFFFFFFFF) | 1
        q = f32(f32(float(bits)) / umax)
        out.append(f32(f32(q * 2.0) - 1.0))
    return out


def scan_map(coords, offsets):
    """Brute-force Scan builder: first (lowest) matching row, -1 on negative."""
    out = []
    for c in coords:
        for o in offsets:
            n = [c[1] + o[0], c[2] + o[1], c[3] + o[2]]
            found = -1
            if min(n) >= 0:
                for r, d in enumerate(coords):
                    if d[0] == c[0] and [d[1], d[2], d[3]] == n:
                        found = r
                        break
            out.append(found)
    return out


def main():
    json.dump({"source": "sparse_decoder_tests.rs:189-236", "coords": [[0, 0, 0, 0], [0, 1, 0, 0]],
               "input": [1.0, 2.0], "weight": [10.0, 1.0, 100.0], "bias": [0.0],
               "kernel": [3, 1, 1], "expected": [201.0, 12.0]},
              open(os.path.join(HERE, "kat_neighbor_voxels.json"), "w"), indent=1)
    json.dump({"source": "sparse_decoder_tests.rs:238-292", "coords": [[0, 0, 0, 0], [0, 1, 0, 0]],
               "kernel": [3, 1, 1], "full_row0": [-1, 0, 1], "chunk_rows": [-1, 0, -1]},
              open(os.path.join(HERE, "kat_halo_chunk.json"), "w"), indent=1)
    json.dump({"source": "burn_flex_gmm/src/lib.rs:764-778", "seed": 42, "values": lcg_values(42, 64)},
              open(os.path.join(HERE, "lcg_seed42.json"), "w"), indent=1)
    coords = [[0, x, 0, 0] for x in range(128)] + [[0, 17, 0, 0], [0, 32, 0, 0], [0, 17, 0, 0],
                                                    [0, 32, 0, 0]]
    # 3x3x1 kernel, axis identity: offsets (dx, dy, 0) in kd-major order
    offsets = [[dx, dy, 0] for dx in (-1, 0, 1) for dy in (-1, 0, 1)]
    json.dump({"source": "burn_flex_gmm/src/wgpu/tests.rs:1801-1853", "kernel": [3, 3, 1],
               "coords": coords, "expected_lowest": scan_map(coords, offsets)},
              open(os.path.join(HERE, "dup_coords.json"), "w"))


if __name__ == "__main__":
    main()

"""Regenerate tests/golden/conformance_golden.json from the reference sources.

Run where a needle-cs source tree is available, passing its path:

    python tests/golden/make_golden.py NEEDLE_CS_ROOT

Two sources feed the fixture:
  * "fixtures": the golden math truths printed by the reference's own
    tools/conformance_fixtures.py `golden()` (imported and executed here).
  * "csharp_asserts": the literal expectations that the reference's xUnit
    conformance suite hard-codes, transcribed with their file:line so that a
    reader can check them against tests/Needle.Tests/Conformance/
    KernelConformanceTests.cs.

The GPU box does not have the reference tree; the tests read only the JSON.
"""
import contextlib
import importlib.util
import io
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference_fixtures(root):
    path = os.path.join(root, "tools", "conformance_fixtures.py")
    spec = importlib.util.spec_from_file_location("needle_conformance_fixtures", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        module.golden()
    return json.loads(out.getvalue()), module.ENTRIES


CSHARP_ASSERTS = {
    # KernelConformanceTests.cs:1022-1037 SoftmaxGolden (|err| <= 1e-6)
    "SoftmaxGolden": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1022-1037",
                      "input": [1.0, 2.0, 3.0], "expected": [0.09003057, 0.24472848, 0.66524094],
                      "uniform_input": [0.0, 0.0, 0.0], "uniform_expected": 0.33333334, "tol": 1e-6},
    # KernelConformanceTests.cs:1061-1071 DotGolden
    "DotGolden": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1061-1071", "expected": 120.0},
    # KernelConformanceTests.cs:1137-1156 QuantizeInt8Golden
    "QuantizeInt8Golden": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1137-1156",
                           "input": [-4.0, 0.0, 4.0, 0.0, 0.0, 0.0, 0.0, 0.0],
                           "scale": 0.03149606, "scale_tol": 1e-6,
                           "bytes": [-127, 0, 127, 0, 0, 0, 0, 0]},
    # KernelConformanceTests.cs:1174-1188 SinkhornGolden (not on the int8 decode path; recorded for completeness)
    "SinkhornGolden": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1174-1188",
                       "expected": 0.25},
    # KernelConformanceTests.cs:1310-1330 ArgMaxMaskedGolden
    "ArgMaxMaskedGolden": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1310-1330",
                           "x": "x[i] = i for i < 64", "mask_single": [0, 32], "expected_single": 37,
                           "mask_empty": [0, 0], "expected_empty": -1,
                           "tie_value": 2.0, "mask_full": [4294967295, 4294967295], "expected_tie": 0},
    # KernelConformanceTests.cs:1356-1362 BestProbabilityGolden
    "BestProbabilityGolden": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1356-1362",
                              "values": [1.0, 2.0, 3.0], "best": 3.0, "expected": 0.66524094, "tol": 1e-6},
    # KernelConformanceTests.cs:1336-1353 BestProbability(count=1) must be exactly 1
    "BestProbabilityCountOne": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1350-1353",
                                "expected": 1.0},
    # Conformance/KernelConformanceTests.cs:1262-1285 ArgMaxMasked theory rows (length, pattern)
    "ArgMaxMaskedCases": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1287-1303",
                          "seed": 0x0A969, "fill_scale": 5.0,
                          "cases": [[0, 0], [1, 1], [31, 1], [32, 1], [33, 2], [64, 2], [100, 1], [100, 3],
                                    [8192, 2], [8192, 0]]},
    # AttentionTileConformance theory rows (kvHeads, heads, first, count, capture); tolerance 5e-5*peak,
    # probabilities 1e-5 (KernelConformanceTests.cs:399-485)
    "AttentionTileCases": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:399-485",
                           "positions": 45, "out_tol_rel_peak": 5e-5, "prob_tol": 1e-5,
                           "cases": [[2, 6, 0, 45, True], [2, 6, 13, 32, True], [2, 6, 41, 4, True],
                                     [8, 1, 0, 45, True], [1, 6, 0, 1, False], [2, 6, 7, 2, False]]},
    # MergePartialsConformance (count, heads); |err| <= 1e-6 (KernelConformanceTests.cs:494-560)
    "MergePartialsCases": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:494-560",
                           "cases": [[1, 1], [1, 6], [2, 1], [2, 6], [3, 6]], "tol": 1e-6},
    # MatMulConformance shapes (bits, rows, cols, tokens), seed 0x9ABC; |err| <= 1e-3*max(1,|expected|)
    "MatMulCases": {"cite": "tests/Needle.Tests/Conformance/KernelConformanceTests.cs:51-185",
                    "golden": [[0x1234, 2, 4, 128, 2], [0x1234, 4, 4, 128, 2]],
                    "shapes": [[2, 5, 768, 1], [2, 5, 768, 3], [4, 7, 384, 5], [2, 3, 128, 8], [4, 97, 768, 3],
                               [2, 5, 768, 0]],
                    "range_odd": [0x9ABC, 2, 8, 128, 3, 3, 7], "tol": 1e-3},
}


def main(argv):
    if len(argv) < 2:
        raise SystemExit("usage: make_golden.py NEEDLE_CS_SOURCE_TREE  (the needle-cs checkout to read fixtures from)")
    root = argv[1]
    fixtures, entries = load_reference_fixtures(root)
    doc = {
        "generated_by": "tests/golden/make_golden.py",
        "source": "needle-cs tools/conformance_fixtures.py golden() + KernelConformanceTests.cs literals",
        "fixtures": fixtures,
        "entries": entries,
        "csharp_asserts": CSHARP_ASSERTS,
    }
    out = os.path.join(HERE, "conformance_golden.json")
    with open(out, "w") as f:
        json.dump(doc, f, indent=1, sort_keys=True)
    print("wrote", out)


if __name__ == "__main__":
    main(sys.argv)

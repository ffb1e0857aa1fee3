"""Copy the reference's XGBoost 3.4.1 golden vectors into tests/golden/.

The reference (mdai001/FerrisBoost) ships little-endian float32 fixtures that
pin its CPU engine bit for bit against XGBoost 3.4.1
(tests/bit_exact_vs_xgboost.rs:213-554 of the reference).  They are data, not
code: `<case>.x` (row-major features), `<case>.y` (labels), `<case>.w`
(sample weights, weighted/monotone sets only), `<case>.margin` (expected raw
margins) and the three index files describing each case's parameters.

Run once in a container that has the reference mounted:
    python tests/golden/make_golden.py /path/to/reference
The GPU box never needs the reference: the copies travel with the repository.
"""
import pathlib
import shutil
import sys

SUFFIXES = (".x", ".y", ".w", ".margin")
INDEXES = ("index.json", "weighted_index.json", "monotone_index.json")


def main(ref_root: str) -> None:
    src = pathlib.Path(ref_root) / "tests" / "fixtures"
    dst = pathlib.Path(__file__).resolve().parent
    n = 0
    for p in sorted(src.iterdir()):
        if p.name in INDEXES or p.suffix in SUFFIXES:
            shutil.copyfile(p, dst / p.name)
            n += 1
    print(f"copied {n} fixture files into {dst}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")

"""Regenerates the golden fixtures in this folder from a checkout of the reference
(JakeATX/sj-kvarn-codec): the directory named by SJK_REF_DIR, else a `reference` checkout
beside this repository. The fixtures are committed, so running the tests never needs the
reference.

  expected_vectors.txt  the reference's 21 FNV-1a 64 hashes of seal records, decoded
                        rows and tq6_0 staging bytes (its tests/expected_vectors.txt)
  expected_state.txt    the reference's 5 FNV-1a 64 hashes of sequence-state streams
                        (its tests/expected_state.txt)
"""
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("SJK_REF_DIR") or os.path.join(HERE, "..", "..", "..", "reference")


def copy_hashes(name, pattern):
    lines = [ln.rstrip("\n") for ln in open(os.path.join(REF, "tests", name))]
    keep = [ln for ln in lines if re.match(pattern, ln)]
    with open(os.path.join(HERE, name), "w") as f:
        f.write(f"# golden data from the reference's tests/{name} (FNV-1a 64 hashes)\n")
        for ln in keep:
            f.write(ln + "\n")
    return len(keep)


def main():
    n1 = copy_hashes("expected_vectors.txt", r"^(seal|tq6) ")
    n2 = copy_hashes("expected_state.txt", r"^state ")
    print(f"expected_vectors.txt: {n1} lines, expected_state.txt: {n2} lines")


if __name__ == "__main__":
    main()

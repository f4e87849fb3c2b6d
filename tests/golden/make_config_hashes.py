"""Regenerates config_hashes.txt: SHA-256 digests (first 32 hex digits) of the record bytes the reference produces at
the benchmark configurations' own shapes and seeds, from the seeded generator's rows (sj-kvarn-codec_b200/csrc/
sjk_synth.h, host build). bench.py prints them beside the GPU's digests when it runs without its CPU legs, and
tests/test_config_golden.py re-derives them from the compiled reference (oracle/_ref) when it is present.

  config0_records   the 128 records of config 0's 4096-token commit (4/4, seed 0), sealed by sj_kvarn_layer_seal
  config2_records   the 128 records of config 2's commit (3/2 trellis, K Student-t(4), seed 2), same schedule

Needs oracle/_ref/libsjref.so (the reference compiled from its own source: `make -C oracle SJK_REF_DIR=...`).
"""
import hashlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.join(HERE, "..", "..")
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "sj-kvarn-codec_b200")):
    sys.path.insert(0, p)

import refcache  # noqa: E402

D, H = 256, 4


def commit_records(seed, bits, heavy, threaded=False):
    """The config-0 schedule on the reference: 8,320 positions through the policy in ubatches of 512 (tail 4096 ->
    8192, n_ctx 16384), then the commit begin_ubatch(8320) asks for (B 128 -> 4224)."""
    rl = refcache.RefLayer(D, H, 16384, 512, bits_k=bits[0], bits_v=bits[1], tail=4096, tail_max=8192)
    scale = refcache.synth_scales(seed, 0, 1, H, D, lib=rl.R)[0]
    pos = 0
    while pos < 8320:
        n = min(512, 8320 - pos)
        rl.begin_ubatch(pos, n, threaded)
        k, v = refcache.synth_kv(seed, 0, H, D, heavy, scale, pos, n, lib=rl.R)
        rl.store(pos, k, v)
        pos += n
    rl.begin_ubatch(8320, 512, threaded)
    assert rl.pol.B == 4224
    recs = rl.records(0, 32)
    rl.close()
    return recs


def digest(a):
    return hashlib.sha256(a.tobytes()).hexdigest()[:32]


def compute():
    return {"config0_records": digest(commit_records(0, (4, 4), False)),
            "config2_records": digest(commit_records(2, (3, 2), True, threaded=True))}


def main():
    out = compute()
    with open(os.path.join(HERE, "config_hashes.txt"), "w") as f:
        f.write("# SHA-256 (first 32 hex digits) of reference record bytes at the benchmark configurations "
                "(make_config_hashes.py)\n")
        for k, v in out.items():
            f.write(f"{k} {v}\n")
    print(out)


if __name__ == "__main__":
    main()

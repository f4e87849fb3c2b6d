"""The committed reference digests of the configurations' records (tests/golden/config_hashes.txt): re-derived by the
oracle restatement (always) and by the compiled reference (when oracle/_ref is built), from the seeded generator's
rows. Pins the oracle at the benchmark shapes, and the fixture that bench.py prints beside the GPU's digests."""
import hashlib
import os

import numpy as np
import pytest

import refcache

HERE = os.path.dirname(os.path.abspath(__file__))
D, H = 256, 4


def _golden():
    out = {}
    for ln in open(os.path.join(HERE, "golden", "config_hashes.txt")):
        f = ln.split()
        if len(f) == 2 and not ln.startswith("#"):
            out[f[0]] = f[1]
    return out


def _digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:32]


def _oracle_commit(oracle_lib, seed, bits, heavy):
    O = oracle_lib.lib()
    trellis = bits != (4, 4)
    oc = oracle_lib.OracleCache(D, H, bits[0], bits[1], trellis, 16, 0, True, 128, 4096, 8192, 512, 16384)
    pol = oracle_lib.Policy()
    O.ora_policy_init(pol, 128, 4096, 8192, 128, 0)
    scale = refcache.synth_scales(seed, 0, 1, H, D, lib=O)[0]
    for pos in range(0, 8320, 512):
        n = min(512, 8320 - pos)
        O.ora_policy_begin(pol, pos, n)
        if pol.B_pending > pol.B:
            oc.seal(pol.B, pol.B_pending)
        O.ora_policy_commit(pol)
        k, v = refcache.synth_kv(seed, 0, H, D, heavy, scale, pos, n, lib=O)
        kr, vr = oracle_lib.fwht_rows(k), oracle_lib.fwht_rows(v)
        for i in range(n):
            oc.store(pos + i, kr[i], vr[i])
    O.ora_policy_begin(pol, 8320, 512)
    assert (pol.B, pol.B_pending) == (128, 4224)
    oc.seal(pol.B, pol.B_pending)
    recs = oc.body_bytes(32)
    oc.close()
    return recs


@pytest.mark.parametrize("name,seed,bits,heavy", [("config0_records", 0, (4, 4), False),
                                                  ("config2_records", 2, (3, 2), True)])
def test_oracle_reproduces_config_digests(oracle_lib, name, seed, bits, heavy):
    assert _digest(_oracle_commit(oracle_lib, seed, bits, heavy)) == _golden()[name]


@pytest.mark.skipif(not refcache.available(), reason="reference not compiled here")
def test_reference_reproduces_config_digests():
    import sys
    sys.path.insert(0, os.path.join(HERE, "golden"))
    import make_config_hashes
    assert make_config_hashes.compute() == _golden()

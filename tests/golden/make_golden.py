"""Generate the golden fixtures from the reference's own code.

Run here, where the reference tree exists (it is absent on GPU boxes):

    make -C oracle REF_DIR=<reference tree> && python tests/golden/make_golden.py

The reference's tests keep no golden files: their goldens are seeded input
generators plus fp64 references (verify_kernel.cpp).  This script replays
those seeded cases through the reference's own transcription, compiled from
its sources into oracle/_ref/libfufft_ref.so, and records
  * reference_cases.npz     full input/output arrays of the small cases;
  * reference_digests.json  SHA-256 digests of every input and output array of
                            every case (large ones included), plus the
                            reference suite's own verdict.
The tests regenerate the inputs with the oracle's generator, check the input
digests (pins the generator), run the oracle and check the output digests
(pins the oracle bit for bit).
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.oracle import Oracle, Reference  # noqa: E402

CONV_CASES = [(8, 1, 3), (8, 4, 8), (64, 1, 3), (64, 8, 16), (128, 1, 8), (256, 1, 4), (256, 4, 8),
              (512, 1, 2), (512, 8, 16), (1024, 1, 4), (2048, 1, 2), (4096, 1, 2)]
BFP_CASES = [(512, 0), (512, 1), (4096, 0), (4096, 1)]
R2_CASES = [(512, 1, 4), (512, 8, 8), (256, 1, 4)]
TWOD_CASES = [(64, 64, 3), (8, 512, 2), (512, 8, 2)]
LARGE_CASES = [(32768, 2, 8, 4096, False), (32768, 2, 8, 4096, True), (32768, 2, 16, 2048, True),
               (131072, 1, 16, 8192, True), (524288, 1, 16, 2048, True)]
SMALL = 4096  # store full arrays when the case has at most this many points


def digest(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def main() -> None:
    o, r = Oracle(), Reference()
    arrays, dig = {}, {"suite_all_pass": r.L.ref_run_suite() == 0}

    def record(key, small, **kv):
        dig[key] = {k: digest(v) for k, v in kv.items()}
        if small:
            for k, v in kv.items():
                arrays[f"{key}/{k}"] = v

    for n, cpb, batch in CONV_CASES:
        a, b = r.gen_test(n, cpb, batch)
        b8 = o.permute_dr(b, n, 8)
        rec = dict(a=a, b=b, ip=r.pipeline_ip(a, b8, n, cpb),
                   fused=r.pipeline_fused(a, o.bperm(b8, n, 8), n, cpb),
                   fwd=r.pipeline_fwd(a, n, cpb))
        rec["apply"] = r.pipeline_apply(rec["fwd"], b8, n, cpb)
        if o.factorise(n, 16)[1] >= 1:
            b16 = o.permute_dr(b, n, 16)
            rec["v16"] = r.pipeline_v16(a, b16, n, cpb if (n // 16) % cpb == 0 else 1)
            rec["v16f"] = r.pipeline_v16f(a, o.bperm(b16, n, 16), n, 1)
            if (n // 8) * cpb % 32 == 0:
                rec["r16"] = r.pipeline_r16(a, b16, n, cpb)
        record(f"conv/{n}/{cpb}/{batch}", n * batch <= SMALL, **rec)

    for n, seed in BFP_CASES:
        a, b = r.gen_bfp(n, seed)
        b16 = o.permute_dr(b, n, 16)
        aq, as_ = r.bfp_quantize(a)
        bq, bs = r.bfp_quantize(b16)
        oq, os_ = r.v16_bfp(aq, as_, bq, bs, n)
        record(f"bfp/{n}/{seed}", True, a=a, b=b, aq=aq, a_scale=np.float32([as_]), bq=bq,
               b_scale=np.float32([bs]), oq=oq, o_scale=np.float32([os_]))

    for n, cpb, batch in R2_CASES:
        xr, yr, h, b_dr = r.gen_r2(n, batch)
        ur, vr = r.conv_r2(xr, yr, b_dr, n, cpb)
        record(f"r2/{n}/{cpb}/{batch}", True, xr=xr, yr=yr, h=h, b_dr=b_dr, ur=ur, vr=vr)

    for h, w, batch in TWOD_CASES:
        a, b = r.gen_2d(h, w, batch)
        rows = np.array([o.chain_rev(i, o.chain(h, 8)) for i in range(h)])
        cols = np.array([o.chain_rev(i, o.chain(w, 8)) for i in range(w)])
        bb = b.reshape(batch, h, w)
        b2 = np.ascontiguousarray(bb[:, rows][:, :, cols]).ravel()
        record(f"conv2d/{h}/{w}/{batch}", False, a=a, b=b, b_dr=b2, out=r.conv2d(a, b2, h, w))

    for n, batch, r_out, mid, v16 in LARGE_CASES:
        a, b = r.gen_large_cfg(n, batch, r_out, mid)
        chain = o.foursteps_chain(n, r_out, mid, 16 if v16 else 8)
        rev = o.rev_table(chain, n)
        b_dr = np.ascontiguousarray(b.reshape(batch, n)[:, rev]).ravel()
        record(f"large/{n}/{batch}/{r_out}/{mid}/{int(v16)}", False, a=a, b=b, b_dr=b_dr,
               four=r.foursteps_cfg(a, b_dr, n, r_out, mid, v16),
               mono=r.monolithic_cfg(a, b_dr, n, r_out, mid, v16))

    np.savez_compressed(os.path.join(HERE, "reference_cases.npz"), **arrays)
    with open(os.path.join(HERE, "reference_digests.json"), "w") as f:
        json.dump(dig, f, indent=1, sort_keys=True)
    print(f"{len(arrays)} arrays, {len(dig)} cases; reference suite all pass: {dig['suite_all_pass']}")


if __name__ == "__main__":
    main()

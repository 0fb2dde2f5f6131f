"""One rank of the C++ decomposed driver (b200dp_dd_*) in its own process and on
its own GPU, for tests/test_gpu_dd.py.

Rank 0 makes the NCCL group id and writes it to a file that the other ranks
wait for; every rank builds its engine on GPU `rank`, runs the requested
work and saves its owned atoms' ids, positions, velocities and forces plus
the global energy, virial and thermodynamic state.  No torch on this path.
"""
import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "dpa4c-scale-aware-md_b200"))

import b200dp  # noqa: E402
import systems  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--nranks", type=int, required=True)
    ap.add_argument("--grid", type=int, nargs=3, required=True)
    ap.add_argument("--model", required=True)
    ap.add_argument("--mol", type=int, nargs=3, required=True, help="water molecules per axis, or FCC cells")
    ap.add_argument("--system", default="water", choices=["water", "cu"])
    ap.add_argument("--ensemble", default="nvt", choices=["nvt", "npt"])
    ap.add_argument("--idfile", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--precision", default="fp64")
    ap.add_argument("--md-steps", type=int, default=0)
    ap.add_argument("--rebuild-every", type=int, default=5)
    ap.add_argument("--halo", type=float, default=8.0)
    a = ap.parse_args()
    s = systems.water(*a.mol) if a.system == "water" else systems.fcc(a.mol[0])
    if a.rank == 0:
        uid = b200dp.dd_unique_id()
        tmp = a.idfile + ".tmp"
        with open(tmp, "wb") as f:
            f.write(uid)
        os.replace(tmp, a.idfile)
    else:
        t0 = time.time()
        while not os.path.exists(a.idfile):
            if time.time() - t0 > 120:
                raise SystemExit("no group id")
            time.sleep(0.05)
        uid = open(a.idfile, "rb").read()
    prec = b200dp.FP64 if a.precision == "fp64" else b200dp.MIXED
    dp = b200dp.DeepPot(a.model, precision=prec, device=a.rank)
    dd = b200dp.DD(dp, uid, a.nranks, a.rank, s.coord, s.atype, s.box, a.grid, halo=a.halo, max_polls=1 << 26)
    out = {}
    dd.force()
    e, v = dd.result()
    ids, x, _, f = dd.owned()
    out.update(energy=e, virial=v, ids=ids, force=f)
    if a.md_steps:
        sys.path.insert(0, HERE)
        from test_gpu_dd import md_setup

        masses, vel, kw = md_setup(s, a.system, a.ensemble)
        dd.md_start(masses, vel=vel, rebuild_every=a.rebuild_every, **kw)
        dd.md_run(a.md_steps)
        th = dd.thermo()
        ids, x, vv, f = dd.owned()
        out.update(md_ids=ids, md_x=x, md_v=vv, md_f=f, thermo=np.array([th[k] for k in dd.THERMO]))
    np.savez(a.out, **out)
    dd.close()
    dp.close()


if __name__ == "__main__":
    main()

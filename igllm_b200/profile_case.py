"""A small verify-round case for kernel profilers.

    python -m igllm_b200.profile_case [--vocab 32768] [--k 4] [--rounds 3] [--context 1024]

The E2B layer stack at full width (35 layers, hidden 1536, FFN 6144, head 256,
window 512, key/value sharing) with a reduced vocabulary, so the per-layer
kernels are the decode path's own while the device holds about 1.3 GB.  The
session is primed to `context` ids (prime passes run before profiling
starts), then `rounds` verify rounds of `k` lanes run between
cuProfilerStart and cuProfilerStop: a profiler started with
--profile-from-start off sees those launches only.
"""

import argparse
import ctypes

import numpy as np

import igllm_b200 as ig


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--vocab", type=int, default=32768)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--context", type=int, default=1024)
    args = ap.parse_args()

    spec = ig.spec_e2b(seed=1, window_limit=4096)
    spec.vocab = args.vocab
    model = ig.Model(spec=spec, device=0, window_limit=4096)
    sess = ig.Session(model)
    rng = np.random.default_rng(0)
    sess.prime(rng.integers(0, args.vocab, args.context).astype(np.int32))
    blocks = rng.integers(0, args.vocab, (args.rounds, args.k)).astype(np.int32)
    sess.bench(blocks[:1], args.k)  # captures the pass of this shape
    cu = ctypes.CDLL("libcuda.so.1")
    cu.cuProfilerStart()
    ms, _ = sess.bench(blocks, args.k)
    cu.cuProfilerStop()
    print(f"{args.rounds} rounds of {args.k} lanes at context {args.context}: {1000 * ms / args.rounds:.1f} us/round")
    sess.close()
    model.close()


if __name__ == "__main__":
    main()

"""Seeded synthetic workloads with the benchmark configurations' shapes.

Config 3 (chunked prefill): 32 prompts of ~U[100, 800] tokens prefilled in
256-token chunks; round r holds the r-th chunk of every prompt that has one.
Config 5 (1.7B decode): 512 sequences with contexts ~log-U[64, 4096].
"""
import numpy as np


def uniform_lens(seed, n, lo, hi):
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n)


def loguniform_lens(seed, n, lo, hi):
    r = np.random.default_rng(seed)
    return np.exp(r.uniform(np.log(lo), np.log(hi), size=n)).astype(np.int64)


def config5_context_lens(seed=0, n=512, lo=64, hi=4096):
    return loguniform_lens(seed, n, lo, hi)


def config3_rounds(seed=0, n=32, lo=100, hi=800, chunk=256):
    """Prompt lengths ~U[lo, hi]; round r prefills tokens [chunk r, chunk r + chunk) of each."""
    lens = uniform_lens(seed, n, lo, hi)
    rounds = []
    r = 0
    while True:
        start = r * chunk
        active = [i for i in range(n) if lens[i] > start]
        if not active:
            break
        rounds.append([(i, start, int(min(chunk, lens[i] - start))) for i in active])
        r += 1
    return lens, rounds

"""Host-side Sampler: mirror of generator.Sampler (src/generator.zig:65-127, 338-463).

Repeat counts over the last ``repeat_last_n`` tokens, the penalised greedy
pick for temperature <= 0, top-k insertion, exp((l - max) / T), the top-p
cut and the cumulative draw.  The PRNG is xoshiro256++ seeded through
SplitMix64 (the published generator behind Zig's std.Random.DefaultPrng) with
a float(f32) built from 23 mantissa bits and a leading-zero exponent; no Zig
toolchain exists here to pin sampled streams bit for bit against the
reference, only the pure helpers are pinned by its tests.
"""

from __future__ import annotations

import numpy as np

from .errors import VvliError

_M64 = (1 << 64) - 1


def validate_options(o) -> None:  # validateSamplingOptions (:338-342)
    if o.temperature < 0.0 or o.temperature != o.temperature:
        raise VvliError("InvalidSamplingOptions")
    if o.top_p <= 0.0 or o.top_p > 1.0 or o.top_p != o.top_p:
        raise VvliError("InvalidSamplingOptions")
    if o.repeat_penalty < 1.0 or o.repeat_penalty != o.repeat_penalty:
        raise VvliError("InvalidSamplingOptions")


class Xoshiro256:
    def __init__(self, seed: int):
        s = seed & _M64
        self.s = []
        for _ in range(4):
            s = (s + 0x9E3779B97F4A7C15) & _M64
            z = s
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
            self.s.append(z ^ (z >> 31))

    @staticmethod
    def _rotl(x, k):
        return ((x << k) | (x >> (64 - k))) & _M64

    def next(self) -> int:
        s = self.s
        r = (self._rotl((s[0] + s[3]) & _M64, 23) + s[0]) & _M64
        t = (s[1] << 17) & _M64
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = self._rotl(s[3], 45)
        return r

    def float32(self) -> float:
        rand = self.next()
        lz = 64 - rand.bit_length()
        if lz >= 41:
            lz = 41 + (64 - self.next().bit_length())
            if lz == 41 + 64:
                lz += 32 - ((self.next() & 0xFFFFFFFF) | 0x7FF).bit_length()
        mantissa = rand & 0x7FFFFF
        bits = ((126 - lz) << 23) | mantissa
        return float(np.array([bits], dtype=np.uint32).view(np.float32)[0])


def repeat_counts(n, prompt, generated, o) -> np.ndarray:  # buildRepeatCounts (:344-360)
    counts = np.zeros(n, dtype=np.uint32)
    if o.repeat_penalty <= 1.0 or o.repeat_last_n == 0:
        return counts
    seq = list(prompt) + list(generated)
    for tok in seq[max(0, len(seq) - o.repeat_last_n):]:
        if tok < n and counts[tok] != 0xFFFF:
            counts[tok] += 1
    return counts


def adjusted(logits: np.ndarray, counts: np.ndarray, rp: float) -> np.ndarray:  # adjustedLogit (:399-402)
    lg = np.asarray(logits, dtype=np.float32)
    if rp <= 1.0:
        return lg.copy()
    rp32 = np.float32(rp)
    pen = np.where(lg < 0, lg * rp32, lg / rp32).astype(np.float32)
    return np.where(counts > 0, pen, lg).astype(np.float32)


def first_argmax(v: np.ndarray) -> int:
    """llm.argmax (src/llm.zig:778-789): first index of the maximum (NaN never wins)."""
    return int(np.argmax(np.where(np.isnan(v), -np.inf, v))) if v.size else 0


class Sampler:
    def __init__(self, vocab_size: int, options):
        seed = options.seed
        if seed is None:
            seed = int.from_bytes(np.random.default_rng().bytes(8), "little")
        if seed == 0:
            seed = 0x9E3779B97F4A7C15
        self.vocab_size = vocab_size
        self.rng = Xoshiro256(seed)

    def next(self, logits, prompt, generated, o) -> int:  # Sampler.next (:97-126)
        validate_options(o)
        lg = np.asarray(logits, dtype=np.float32)
        counts = repeat_counts(lg.size, prompt, generated, o)
        scores = adjusted(lg, counts, o.repeat_penalty)
        if o.temperature <= 0.0:
            return first_argmax(scores)
        finite = np.isfinite(scores)
        ids = np.nonzero(finite)[0]
        if ids.size == 0:
            return first_argmax(lg)
        limit = ids.size if o.top_k == 0 else min(o.top_k, lg.size)
        # insertTopCandidate keeps, among equal logits, the earliest ids
        order = np.lexsort((ids, -scores[ids]))
        cand = ids[order][:limit]
        cl = scores[cand].astype(np.float32)
        t = np.float32(max(o.temperature, 1e-6))
        probs = np.exp(((cl - cl[0]) / t).astype(np.float32)).astype(np.float32)
        probs = np.where(np.isfinite(probs), probs, np.float32(0)).astype(np.float32)
        total = np.float32(0)
        for p in probs:
            total = np.float32(total + p)
        if total <= 0 or not np.isfinite(total):
            return int(cand[0])
        count = cand.size
        if o.top_p < 1.0:
            cum = np.float32(0)
            for i, p in enumerate(probs):
                cum = np.float32(cum + p)
                if cum / total >= np.float32(o.top_p):
                    count = i + 1
                    break
        cand, probs = cand[:count], probs[:count]
        tot = np.float32(0)
        for p in probs:
            tot = np.float32(tot + p)
        if tot <= 0 or not np.isfinite(tot):
            return int(cand[0])
        target = np.float32(min(self.rng.float32(), 0.99999994)) * tot
        cum = np.float32(0)
        for c, p in zip(cand, probs):
            cum = np.float32(cum + p)
            if target <= cum:
                return int(c)
        return int(cand[-1])


class DeviceSampler:
    """generator.Sampler whose next() runs on the GPU (vvli_cuda_sample).

    Seeding follows Sampler.init (src/generator.zig:74-90): a random seed when
    none is given, 0 replaced by 0x9e3779b97f4a7c15, SplitMix64 into the
    xoshiro256++ state, which then lives here between calls.
    """

    def __init__(self, vocab_size: int, options):
        seed = options.seed
        if seed is None:
            seed = int.from_bytes(np.random.default_rng().bytes(8), "little")
        if seed == 0:
            seed = 0x9E3779B97F4A7C15
        self.vocab_size = vocab_size
        self.state = np.array(Xoshiro256(seed).s, dtype=np.uint64)

    def next(self, runner, prompt, generated, o) -> int:  # Sampler.next (:97-126)
        validate_options(o)
        n = int(o.repeat_last_n)
        recent = list(prompt) + list(generated)
        return runner.sample(o, recent[max(0, len(recent) - n):] if n else [], self.state)

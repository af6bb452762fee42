"""Pins the sampler restatement (oracle/tokenizer_ref.py), the checker of the
device sampler, against a second, independent restatement of sampler.rs
written here as scalar f32 loops that follow the Rust line by line
(softmax :28-39, sample_argmax :67-79, random_f32 :81-91, sample_mult
:93-104, sample_topp :117-155 with its persistent probability_idx array and
the stable sort_by of the whole array, sample :157-180). The reference has no
sampler tests or golden vectors to pin against. CPU only."""
from __future__ import annotations

import functools

import numpy as np
import pytest

import tokenizer_ref as tr

F = np.float32


def exp32(x: np.float32) -> np.float32:
    return F(np.exp(np.float64(x)))  # e^x rounded once to f32 (the exp the device uses)


class LoopSampler:
    def __init__(self, vocab: int, temperature: float, top_p: float, seed: int):
        self.n = vocab
        self.temperature, self.top_p = F(temperature), F(top_p)
        self.seed = seed
        self.idx = [[F(0.0), 0] for _ in range(vocab)]  # probability_idx: {prob, index}

    @staticmethod
    def random_f32(seed: int) -> np.float32:
        m = (1 << 64) - 1
        st = seed & m
        st ^= st >> 12
        st ^= (st << 25) & m
        st ^= st >> 27
        r = ((st * 0x2545F4914F6CDD1D) & m) >> 32
        return F(F(r >> 8) / F(16777216.0))

    @staticmethod
    def argmax(p) -> int:
        mi, mp = 0, p[0]
        for i in range(1, len(p)):
            if p[i] > mp:
                mi, mp = i, p[i]
        return mi

    @staticmethod
    def softmax(x) -> None:
        mx = F(-np.inf)
        for v in x:
            mx = max(mx, v) if v == v else mx
        s = F(0.0)
        for i in range(len(x)):
            x[i] = exp32(F(x[i] - mx))
            s = F(s + x[i])
        for i in range(len(x)):
            x[i] = F(x[i] / s)

    def sample(self, logits) -> int:
        x = [F(v) for v in logits]
        if self.temperature == F(0.0):
            return self.argmax(x)
        for q in range(self.n):
            x[q] = F(x[q] / self.temperature)
        self.softmax(x)
        rnd = self.random_f32(self.seed)
        if self.top_p <= F(0.0) or self.top_p >= F(1.0):
            cdf = F(0.0)
            for i, p in enumerate(x):
                cdf = F(cdf + p)
                if rnd < cdf:
                    return i
            return self.n - 1
        cutoff = F(F(F(1.0) - self.top_p) / F(self.n - 1))
        n0 = 0
        for i, p in enumerate(x):
            if p >= cutoff:
                self.idx[n0] = [p, i]
                n0 += 1

        def cmp(a, b):  # Sampler::compare: descending prob, Equal otherwise
            return -1 if a[0] > b[0] else (1 if a[0] < b[0] else 0)
        self.idx.sort(key=functools.cmp_to_key(cmp))  # stable, the whole array
        cum = F(0.0)
        last = n0 - 1
        for i in range(n0):
            cum = F(cum + self.idx[i][0])
            if cum > self.top_p:
                last = i
                break
        r = F(rnd * cum)
        cdf = F(0.0)
        for i in range(last + 1):
            cdf = F(cdf + self.idx[i][0])
            if r < cdf:
                return self.idx[i][1]
        return self.idx[last][1]


@pytest.mark.parametrize("temp,top_p", [(0.0, 0.9), (0.7, 0.9), (1.0, 1.0), (0.8, 0.0), (1.3, 0.5), (0.5, 0.999),
                                        (2.0, 0.3)])
def test_vectorized_restatement_equals_loops(temp, top_p):
    V = 257
    rng = np.random.default_rng(int(temp * 100 + top_p * 1000))
    a, b = tr.Sampler(V, temp, top_p, 42), LoopSampler(V, temp, top_p, 42)
    for step in range(8):
        x = (rng.standard_normal(V) * [0.5, 4.0, 1.0, 8.0, 0.1, 3.0, 2.0, 0.02][step]).astype(np.float32)
        if step == 5:  # ties: the lowest index among equal maxima, stable order among equal probabilities
            x[::7] = x.max()
        assert a.sample(x.copy()) == b.sample(x.copy()), (temp, top_p, step)


def test_random_f32_matches_loop_version():
    for seed in (0, 1, 42, 2**63 + 5, 123456789):
        assert tr.random_f32(seed) == LoopSampler.random_f32(seed)

"""Generation loop: the host-side mirror of src/generator.zig.

``generate_greedy`` and ``generate_greedy_measured`` keep the reference's
names, options, results and errors (src/generator.zig:14-48, 142-325).  With
the ``--greedy`` settings (temperature 0, repeat penalty 1.0) the token loop
runs on the GPU through ``Runner.generate_greedy``; other settings run
Sampler.next on the GPU each step (``vvli_b200.sampler.DeviceSampler``) over
logits that never leave the device.
"""

from __future__ import annotations

import dataclasses
import time

from .errors import VvliError
from .runner import Runner
from . import sampler as _sampler


@dataclasses.dataclass
class Options:  # generator.Options (src/generator.zig:14-23)
    max_new_tokens: int = 32
    eos_token_id: int | None = None
    temperature: float = 0.8
    top_p: float = 0.95
    top_k: int = 40
    repeat_penalty: float = 1.10
    repeat_last_n: int = 64
    seed: int | None = None


@dataclasses.dataclass
class Stats:  # generator.Stats (src/generator.zig:25-43)
    prompt_tokens: int
    generated_tokens: int
    prefill_nanoseconds: int
    decode_nanoseconds: int
    total_nanoseconds: int

    def decode_seconds(self) -> float:
        return self.decode_nanoseconds / 1e9 if self.decode_nanoseconds > 0 else 0.0

    def decode_tokens_per_second(self) -> float:
        return _tps(self.generated_tokens, self.decode_nanoseconds)

    def total_tokens_per_second(self) -> float:
        return _tps(self.prompt_tokens + self.generated_tokens, self.total_nanoseconds)


@dataclasses.dataclass
class Result:
    tokens: list
    stats: Stats


def _tps(tokens, ns):
    if tokens == 0 or ns <= 0:
        return 0.0
    return tokens * 1e9 / ns


def generate_greedy(runner: Runner, prompt_tokens, options: Options) -> list:
    """generateGreedy (src/generator.zig:142-175): argmax loop, optional eos."""
    if len(prompt_tokens) == 0:
        raise VvliError("EmptyPrompt")
    tokens, _ = runner.generate_greedy(prompt_tokens, options.max_new_tokens, options.eos_token_id)
    return tokens


def generate_greedy_measured(runner: Runner, prompt_tokens, options: Options) -> Result:
    """generateGreedyMeasured (src/generator.zig:177-293) with the Sampler."""
    if len(prompt_tokens) == 0:
        raise VvliError("EmptyPrompt")
    _sampler.validate_options(options)
    if options.temperature <= 0.0 and (options.repeat_penalty <= 1.0 or options.repeat_last_n == 0):
        tokens, s = runner.generate_greedy(prompt_tokens, options.max_new_tokens, options.eos_token_id)
        return Result(tokens, Stats(s.prompt_tokens, s.generated_tokens, s.prefill_nanoseconds,
                                    s.decode_nanoseconds, s.total_nanoseconds))
    t0 = time.perf_counter_ns()
    runner.prefill(prompt_tokens, 0, logits=False)
    t1 = time.perf_counter_ns()
    smp = _sampler.DeviceSampler(runner.cfg.vocab_size, options)
    out = []
    position = len(prompt_tokens)
    while len(out) < options.max_new_tokens:
        nxt = smp.next(runner, prompt_tokens, out, options)
        out.append(nxt)
        if options.eos_token_id is not None and nxt == options.eos_token_id:
            break
        runner.forward_token(nxt, position, logits=False)
        position += 1
    t2 = time.perf_counter_ns()
    return Result(out, Stats(len(prompt_tokens), len(out), t1 - t0, t2 - t1, t2 - t0))

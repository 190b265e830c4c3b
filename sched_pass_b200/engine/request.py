"""Request state of the serving engine."""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

import numpy as np


class State(enum.Enum):
    WAITING = 0   # arrived, nothing cached
    PREFILL = 1   # prompt partially in the cache
    DECODE = 2    # generating
    DONE = 3


@dataclass(eq=False)  # identity semantics: requests are compared and hashed by object
class Request:
    rid: int
    prompt: np.ndarray            # int32 token ids
    max_new_tokens: int
    arrival: float = 0.0          # seconds (workload clock)
    state: State = State.WAITING
    pages: list = field(default_factory=list)
    cached: int = 0               # tokens whose K/V are in the cache
    output: list = field(default_factory=list)
    token_times: list = field(default_factory=list)  # clock when each output token was produced
    first_scheduled: float | None = None
    urgency: float = 0.0          # control-plane q (0..1)
    tau: int = 0                  # shed budget in tokens (0 = none)
    preemptions: int = 0
    spilled_pages: int = 0        # pages moved to the host KV tier (tiered KV)

    @property
    def prompt_len(self) -> int:
        return int(self.prompt.size)

    @property
    def total_len(self) -> int:
        """Tokens that will be in the cache once the next token is appended."""
        return self.prompt_len + len(self.output)

    @property
    def finished(self) -> bool:
        return len(self.output) >= self.max_new_tokens

    def next_input_token(self) -> int:
        return int(self.output[-1]) if self.output else int(self.prompt[-1])

    def tpot(self) -> float | None:
        """Mean time per output token after the first."""
        if len(self.token_times) < 2:
            return None
        return (self.token_times[-1] - self.token_times[0]) / (len(self.token_times) - 1)

    def ttft(self) -> float | None:
        return (self.token_times[0] - self.arrival) if self.token_times else None

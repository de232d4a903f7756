"""SFStatus: what the runtime knows about a heavy op after it ran.

The same fields and meaning as the reference (src/sf/_status.py:7-65):
``saturated`` outputs that saturated (exact here, since the B200 target
reports sticky per-output events), ``underflow`` outputs where a nonzero
product truncated to 0, ``div0`` / ``invalid`` read off the inputs,
``exact``, and ``outputs_at_max`` the raw count of outputs at +-max.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class SFStatus:
    saturated: int | None = 0
    div0: int = 0
    invalid: int = 0
    exact: bool = False
    outputs_at_max: int = 0
    underflow: int | None = 0

    @property
    def known(self) -> bool:
        return self.saturated is not None and self.underflow is not None

    @property
    def ok(self):
        if self.div0 or self.invalid or self.saturated or self.underflow:
            return False
        if self.saturated is None or self.underflow is None:
            return None
        return True

    def __repr__(self) -> str:
        if self.saturated is None:
            sat = f"saturated=unknown (outputs_at_max={self.outputs_at_max})"
        else:
            sat = f"saturated={'' if self.exact else '<='}{self.saturated}"
        under = "unknown" if self.underflow is None else self.underflow
        return f"SFStatus({sat}, underflow={under}, div0={self.div0}, invalid={self.invalid}, exact={self.exact})"

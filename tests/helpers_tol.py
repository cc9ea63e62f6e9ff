"""The split-K tolerance of docs/splash/dev/tuning/LinearNumerics.hpp:29-126
restated in Python for the GPU tests (pinned to the compiled reference by
tests/test_oracle.py)."""
import math


def ulp_bf16(value: float) -> float:
    mag = abs(value)
    if not (mag >= 2.0 ** -126) or not math.isfinite(mag):
        return 2.0 ** -133
    _, e = math.frexp(mag)
    return 2.0 ** (e - 8)


def silu(v: float) -> float:
    return v / (1.0 + math.exp(-v))


def split_tolerance(epilogue: int, value: float, residual: float, gate: float, up: float, slack: float) -> float:
    b = ulp_bf16(value) + slack
    if epilogue == 1:
        b += ulp_bf16(value - residual)
    if epilogue == 2:
        b += 1.1 * (abs(up) + ulp_bf16(up) + slack) * (ulp_bf16(gate) + slack) + abs(silu(gate)) * (ulp_bf16(up) + slack)
    return b

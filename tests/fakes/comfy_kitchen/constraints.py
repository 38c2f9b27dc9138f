from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class ValidationResult:
    success: bool
    failed_param: str | None = None
    message: str = ""

    @classmethod
    def ok(cls):
        return cls(True)

    @classmethod
    def fail(cls, param, msg=""):
        return cls(False, param, msg)


@dataclass
class FunctionConstraints:
    params: dict = field(default_factory=dict)
    default_devices: tuple = ("cuda", "cpu")
    min_compute_capability: tuple | None = None
    call_rules: tuple = ()

from __future__ import annotations

from .constraints import FunctionConstraints


class BackendRegistry:
    def __init__(self):
        self._backends = {}
        self._priority = []

    def register(self, name, module, constraints):
        self._backends[name] = (module, dict(constraints))
        if name not in self._priority:
            self._priority.append(name)

    def set_priority(self, names):
        self._priority = list(names)

    def get_constraints(self, backend, op):
        entry = self._backends.get(backend)
        return None if entry is None else entry[1].get(op)

    def dispatch(self, op, **kwargs):
        """Call the first backend whose call rules all accept the call."""
        for name in self._priority:
            module, cons = self._backends[name]
            c = cons.get(op)
            if c is None:
                continue
            if all(rule(kwargs).success for rule in c.call_rules):
                return name, getattr(module, op)(**kwargs)
        raise RuntimeError("no backend accepted the call")


registry = BackendRegistry()


def _install_eager():
    from .backends.eager import quantization

    registry.register("eager", quantization, {"int8_linear": FunctionConstraints(params={"x": None})})


_install_eager()

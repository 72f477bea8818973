"""Optional OpenTelemetry spans with a no-op fallback (src/py/mogemma/telemetry.py)."""

from contextlib import AbstractContextManager

from ._typing import trace


class _NoOpSpan:
    def set_attribute(self, _key: str, _value: object) -> None:
        return None


class _NoOpSpanManager(AbstractContextManager[_NoOpSpan]):
    def __enter__(self) -> _NoOpSpan:
        return _NoOpSpan()

    def __exit__(self, *exc: object) -> None:
        return None


class _NoOpTracer:
    def start_as_current_span(self, _name: str) -> AbstractContextManager[_NoOpSpan]:
        return _NoOpSpanManager()


tracer = trace.get_tracer("mogemma_b200") if trace is not None else _NoOpTracer()

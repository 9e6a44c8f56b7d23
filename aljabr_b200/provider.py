"""Provider lifecycle mirroring the reference's compute SPI.

  * ComputeProvider.devices / openSession -- spi/aljabr-spi-compute/src/main/java/
    tech/kayys/aljabr/spi/compute/ComputeProvider.java:16-29
  * ProviderSession.computeBackends / operationSupport / close (idempotent) --
    ProviderSession.java:30-95
  * ComputeRuntime selection by explicit provider id never falls back --
    core/aljabr-compute-runtime/.../ComputeRuntime.java:115-147

The provider id is "andalus/blackwell"; one GPU device per visible B200.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import native

PROVIDER_ID = "andalus/blackwell"
BACKEND_ID = "blackwell"

# operation id -> supported constraint sets (NATIVE) ; everything else UNSUPPORTED
NATIVE_OPERATIONS = {
    "matvec": {"q4_0", "q8_0", "nf4", "q4_k", "q6_k"},
    "matvec.pair": {"q4_0", "q8_0", "q4_k", "q6_k"},
    "matvec.triple": {"q4_0", "q8_0", "q4_k", "q6_k"},
    "matvec.batch": {"q4_0", "q8_0", "q4_k", "q6_k"},
    "dequantize": {"q4_0", "q8_0", "nf4"},
    "attention.gqa.decode": {"f32", "bf16"},
}


@dataclass(frozen=True)
class DeviceDescriptor:
    provider_id: str
    device_id: int
    kind: str
    name: str
    compute_capability: int


@dataclass(frozen=True)
class OperationSupportDescriptor:
    operation_id: str
    support: str            # "NATIVE" | "UNSUPPORTED"
    reason: str | None = None


class ProviderClosed(RuntimeError):
    pass


def operation_support(operation_id: str, constraints: dict) -> OperationSupportDescriptor:
    """NATIVE only for what a kernel implements; never UNKNOWN, never a fallback."""
    if constraints is None:
        raise TypeError("constraints")
    fmt = constraints.get("dtype") or constraints.get("type")
    allowed = NATIVE_OPERATIONS.get(operation_id)
    if allowed is None:
        return OperationSupportDescriptor(operation_id, "UNSUPPORTED", "no Blackwell kernel")
    if fmt is not None and fmt not in allowed:
        return OperationSupportDescriptor(operation_id, "UNSUPPORTED", f"{fmt} not in {sorted(allowed)}")
    return OperationSupportDescriptor(operation_id, "NATIVE", None)


class BlackwellComputeBackend:
    """The backend object a session exposes; it owns nothing itself."""

    def __init__(self, device: DeviceDescriptor):
        self.device = device
        self.closed = False

    def close(self):
        self.closed = True


class BlackwellSession:
    def __init__(self, device: DeviceDescriptor):
        native.call("aljabr_blackwell_init", device.device_id)
        self._device = device
        self._backends = {BACKEND_ID: BlackwellComputeBackend(device)}
        self._closed = False

    def device(self) -> DeviceDescriptor:
        return self._device

    def compute_backends(self) -> dict:
        if self._closed:
            raise ProviderClosed("session is closed")
        return dict(self._backends)

    def operation_support(self, operation_id: str, constraints: dict) -> OperationSupportDescriptor:
        return operation_support(operation_id, constraints)

    def close(self):
        if self._closed:
            return
        self._closed = True
        for b in {id(b): b for b in self._backends.values()}.values():
            b.close()


class BlackwellComputeProvider:
    def descriptor_id(self) -> str:
        return PROVIDER_ID

    def devices(self) -> list:
        L = native.lib()
        out = []
        for d in range(L.aljabr_blackwell_device_count()):
            buf = ctypes.create_string_buffer(256)
            native.check(L.aljabr_blackwell_device_name(buf, 256, d))
            cc = L.aljabr_blackwell_compute_capability(d)
            out.append(DeviceDescriptor(PROVIDER_ID, d, "GPU", buf.value.decode(), cc))
        return out

    def open_session(self, device: DeviceDescriptor) -> BlackwellSession:
        if device.provider_id != PROVIDER_ID:
            raise ValueError(f"device belongs to provider {device.provider_id!r}, not {PROVIDER_ID!r}")
        return BlackwellSession(device)

"""Exception classes with musapy's names and hierarchy.

Mirrors the Python exception mapping of rust/musapy-python/src/error.rs and
the class tree declared in python/musapy/_core.pyi:22-32.
"""


class MusapyError(Exception):
    pass


class DeviceError(MusapyError):
    pass


class DeviceNotConfiguredError(DeviceError):
    pass


class DtypeError(MusapyError):
    pass


class ShapeError(MusapyError):
    pass


class MemoryError(MusapyError):  # noqa: A001 - same name as musapy's class
    pass


class OutOfMemoryError(MemoryError):
    pass


class StreamError(MusapyError):
    pass


class KernelError(MusapyError):
    pass


class InteropError(MusapyError):
    pass


class LinAlgError(MusapyError):
    """Raised by musapy's linalg namespace; exported so that code catching
    it keeps importing (linear algebra itself is not part of this engine)."""

"""tempname_dcu_b200: a B200-native (sm_100a) tensor-parallel compute /
communication overlap framework with the capabilities of Moon-Run/TempName-DCU.

Importing the package has no side effects: torch and the native library are
loaded lazily by the modules that need them.
"""
__version__ = "0.1.0"


def __getattr__(name):
    if name == "FluxB200":
        from .runtime import FluxB200
        return FluxB200
    raise AttributeError(name)

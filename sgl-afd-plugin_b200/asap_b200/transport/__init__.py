"""A<->F transport over NVLink on B200: owner-allocated arenas (CUDA IPC), SM-driven P2P stores, device-written
doorbells and done flags, bounded device waits.  Same exports as the reference's
python/sgl_asap_plugin/transport/__init__.py:21-31.  Submodules load lazily: importing the package or
``layout`` loads neither torch nor libasap."""

import importlib

_EXPORTS = {
    "Geometry": "layout",
    "TransportError": "layout",
    "HandshakeError": "layout",
    "ChannelPoisoned": "layout",
    "AttnChannel": "channel",
    "Ticket": "channel",
    "FfnServer": "server",
    "Job": "server",
    "Row": "server",
}
__all__ = sorted(_EXPORTS)


def __getattr__(name):
    module = _EXPORTS.get(name)
    if module is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    return getattr(importlib.import_module(f"{__name__}.{module}"), name)

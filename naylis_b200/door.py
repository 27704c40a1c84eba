"""Registration of the sm100 backend behind the reference's own dispatch door.

The reference picks its MoM read backend in one module, ``mom_kernels``
(mom_kernels/__init__.py:37-117): ``preflight`` (called by pretrain.py:694-698),
``resolve_mode`` (called once per layer by model.py:164-167), ``mom_read``
(model.py:258-261) and ``announce``. Its callers look those functions up on the
module at every call, so installing a backend is replacing the four functions
with ones that serve mode ``"sm100"`` and hand every other request to the
originals:

    import mom_kernels                       # the reference's package
    from naylis_b200 import door
    door.register(mom_kernels)               # NAYLIS_KERNEL=sm100 selects it

after which the reference's unchanged ``model.py`` and ``pretrain.py`` run
their memory read on this package's kernels whenever ``use_kernel=true``
resolves on a CUDA device and the selection holds. The router stays the
reference's inline code (model.py:178-220); ``naylis_b200.model.MoMLayer`` is
the layer that also runs the fused router.

Selection: by default the environment variable ``NAYLIS_KERNEL=sm100`` (read
at each resolve); ``select=`` takes any zero-argument callable instead. No
fallback crosses the door: a request the sm100 backend takes either resolves
or raises with its reason; a request it does not take goes to the reference's
own branch, unchanged.
"""
from __future__ import annotations

import os

_NAMES = ("preflight", "resolve_mode", "mom_read", "announce")
_SAVED = "_naylis_sm100_originals"


def _device_type(device) -> str:
    t = getattr(device, "type", None)
    return t if isinstance(t, str) else str(device).split(":")[0].lower()


def register(door, backend=None, select=None, device_types=("cuda",)) -> None:
    """Install mode "sm100" into ``door`` (the reference's ``mom_kernels``
    module object). ``backend`` defaults to ``naylis_b200.mom_kernels``;
    ``device_types`` are the device types the backend takes. Registering twice
    replaces the first registration."""
    if backend is None:
        from . import mom_kernels as backend
    if select is None:
        def select():
            return os.environ.get("NAYLIS_KERNEL", "").strip().lower() == backend.MODE
    if hasattr(door, _SAVED):
        unregister(door)
    orig = {name: getattr(door, name) for name in _NAMES}
    setattr(door, _SAVED, orig)

    def wants(device) -> bool:
        return _device_type(device) in device_types and bool(select())

    def preflight(device_type: str) -> None:
        if wants(device_type):
            return backend.preflight(device_type)
        return orig["preflight"](device_type)

    def resolve_mode(device, dtype, *, head_dim=None) -> str:
        if wants(device):
            return backend.resolve_mode(device, dtype, head_dim=head_dim)
        return orig["resolve_mode"](device, dtype, head_dim=head_dim)

    def mom_read(q_sh, k, v, top_idx, top_gates, *, num_blocks, block_size, mode):
        if mode == backend.MODE:
            return backend.mom_read(q_sh, k, v, top_idx, top_gates, num_blocks=num_blocks,
                                    block_size=block_size, mode=mode)
        return orig["mom_read"](q_sh, k, v, top_idx, top_gates, num_blocks=num_blocks,
                                block_size=block_size, mode=mode)

    def announce(name: str) -> None:
        if name == backend.MODE:
            return backend.announce(name)
        return orig["announce"](name)

    for name, fn in zip(_NAMES, (preflight, resolve_mode, mom_read, announce)):
        fn.__doc__ = (orig[name].__doc__ or "") + "\n\n[naylis_b200: mode 'sm100' registered]"
        setattr(door, name, fn)


def unregister(door) -> None:
    """Put the reference's own four functions back."""
    orig = getattr(door, _SAVED, None)
    if orig is None:
        return
    for name, fn in orig.items():
        setattr(door, name, fn)
    delattr(door, _SAVED)


__all__ = ["register", "unregister"]

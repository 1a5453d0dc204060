"""Registers the B200 backend with the reference's Orion as ``backend: b200``.

Orion picks a backend in ``Scheme.setup_backend`` (orion/core/orion.py:100-126)
and validates the name in ``OrionParameters.__post_init__``
(orion/backend/python/parameters.py:122-127).  ``install()`` wraps both:
the validator accepts "b200" and ``setup_backend`` returns a
``B200Library`` for it, leaving every other backend untouched.  Import
orion (the reference checkout on PYTHONPATH) before calling it.
"""
from __future__ import annotations

_installed = False
_factory = None


def install(factory=None) -> None:
    """Register ``backend: b200``.  ``factory`` builds the backend object
    (default: ``B200Library()``); a test may pass a stand-in with the same
    methods."""
    global _installed, _factory
    _factory = factory
    if _installed:
        return
    import orion.core.orion as orion_mod
    from orion.backend.python import parameters

    orig_post = parameters.OrionParameters.__post_init__

    def post_init(self):
        if str(self.backend).lower() == "b200":
            self.backend = "cheddar"
            try:
                orig_post(self)
            finally:
                self.backend = "b200"
        else:
            orig_post(self)

    parameters.OrionParameters.__post_init__ = post_init

    orig_setup = orion_mod.Scheme.setup_backend

    def setup_backend(self, params):
        if params.get_backend() == "b200":
            if _factory is not None:
                lib = _factory()
            else:
                from .library import B200Library
                lib = B200Library()
            lib.setup_bindings(params)
            return lib
        return orig_setup(self, params)

    orion_mod.Scheme.setup_backend = setup_backend
    _installed = True

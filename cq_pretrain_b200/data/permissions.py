"""Image-target permissions of corpus records (reference ``data/loss_permissions.py:3-22``).

A visual may be a generation target only if every owner (the record and the image entry) that
states ``image_loss_allowed`` or ``dcvlm_image_loss_allowed`` allows it: a strict boolean AND.
An absent field keeps the historical default (allowed). A present field must be a real
``bool``; ``None``, numbers and strings raise instead of silently enabling or disabling the
objective, and every field is validated even after a denial. Understanding inputs are never
removed by these flags.
"""

from __future__ import annotations

CONTRACT = "image_loss_boolean_and_v1"
FIELDS = ("image_loss_allowed", "dcvlm_image_loss_allowed")


def image_loss_allowed(*owners) -> bool:
    allowed = True
    for owner in owners:
        for name in FIELDS:
            if name not in owner:
                continue
            value = owner[name]
            if not isinstance(value, bool):
                raise ValueError(f"{name} must be a boolean when present, got {type(value).__name__}")
            allowed = allowed and value
    return allowed

"""Plugin boundary: `get_plugin().build_model(game_spec, config)` returns a
ShrimpNet built from the environment-driven architecture, as the reference's
ShrimpPlugin does (packages/shrimp/python/shrimp/plugin.py:19-76). Only the
model-construction hook belongs to this serve build; training, self-play and
evaluation hooks are not provided."""

from __future__ import annotations

from typing import Any, Mapping

from .model import ShrimpNet


class ShrimpPlugin:
    name = "shrimp"

    def build_model(self, game_spec: Mapping[str, Any], config: Mapping[str, Any]) -> ShrimpNet:
        _ = (game_spec, config)
        return ShrimpNet()


plugin = ShrimpPlugin()


def get_plugin() -> ShrimpPlugin:
    return plugin

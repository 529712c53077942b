"""H3 DMD for B200: a Blackwell-native shared-backbone DMD trainer.

Public entry points: ``python -m h3_a100.entrypoint --config <yaml>`` (CLI),
``h3_a100.api.build_trainer`` (programmatic), ``h3_a100.preflight`` (checks).
"""

__version__ = "0.1.0"
__all__ = ["__version__"]

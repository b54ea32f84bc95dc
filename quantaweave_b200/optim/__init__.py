from .cpu_offload import CPUOffloadAdamW

__all__ = ["CPUOffloadAdamW", "FusedAdamW"]


def __getattr__(name):
    if name == "FusedAdamW":
        from .adamw import FusedAdamW

        return FusedAdamW
    raise AttributeError(name)

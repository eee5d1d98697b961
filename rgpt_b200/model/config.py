"""Attribute-access config mapping (stands in for omegaconf.DictConfig when it is absent)."""
try:  # the reference passes omegaconf.DictConfig objects around; use it when installed
    from omegaconf import DictConfig as _DictConfig  # type: ignore
except Exception:  # pragma: no cover - omegaconf is not installed in this image
    _DictConfig = None


class Config(dict):
    """dict with attribute access and .get, enough for the model/trainer code paths."""

    def __getattr__(self, k):
        try:
            return self[k]
        except KeyError as e:
            raise AttributeError(k) from e

    def __setattr__(self, k, v):
        self[k] = v


def as_config(obj):
    """Config view of a mapping (nested mappings too, so cfg.training.optimizer.lr works on plain dicts)."""
    if _DictConfig is not None and isinstance(obj, _DictConfig):
        from omegaconf import OmegaConf  # type: ignore

        obj = OmegaConf.to_container(obj, resolve=True)
    return Config({k: as_config(v) if isinstance(v, dict) else v for k, v in dict(obj).items()})

"""Model and dataset download from the Hugging Face hub (reference ``axrl/utils/hf/*.py``).

``download_model`` fetches a model repository into ``ModelConfig.get_full_path()`` (resuming /
verifying an existing directory), ``download_data_file`` one dataset file into the data directory
(skipped when it exists).  Both need ``huggingface_hub`` and network access; on a machine without
either they raise with the path that was expected, so a run can instead be pointed at local files.

python -m axrl_b200.utils.hf_download model --name=Qwen/Qwen3-8B
python -m axrl_b200.utils.hf_download data --repo_id=open-r1/DAPO-Math-17k-Processed --filename=all/train-00000-of-00001.parquet
"""

from __future__ import annotations

import logging
import sys
from pathlib import Path

from axrl_b200.configs import AXRL_DIR, HfDataConfig, ModelConfig

logger = logging.getLogger(__name__)


def _hub():  # noqa: ANN202
    try:
        import huggingface_hub
    except ImportError as e:  # pragma: no cover - the image ships it
        raise RuntimeError("huggingface_hub is not installed; place the files locally instead") from e
    return huggingface_hub


def download_model(config: ModelConfig) -> Path:
    target = config.get_full_path()
    logger.info("%s model %s to %s", "verifying" if target.exists() else "downloading", config.name, target)
    try:
        path = _hub().snapshot_download(repo_id=config.name, local_dir=str(target))
    except Exception as e:  # noqa: BLE001
        raise RuntimeError(f"could not download {config.name} to {target}: {e}") from e
    return Path(path)


def download_data_file(config: HfDataConfig) -> Path:
    target = config.get_full_path()
    if target.exists():
        logger.info("data file %s exists, skipping download", target)
        return target
    local = AXRL_DIR.data / config.repo_id
    local.mkdir(parents=True, exist_ok=True)
    try:
        path = _hub().hf_hub_download(repo_id=config.repo_id, filename=config.filename, repo_type="dataset", local_dir=str(local))
    except Exception as e:  # noqa: BLE001
        raise RuntimeError(f"could not download {config.repo_id}/{config.filename} to {target}: {e}") from e
    return Path(path)


def main(argv: list[str] | None = None) -> None:
    from axrl_b200.utils.config_utils import load_and_validate_config

    argv = list(sys.argv[1:] if argv is None else argv)
    what = argv.pop(0) if argv else "model"
    if what == "model":
        download_model(load_and_validate_config(ModelConfig, argv=argv))
    elif what == "data":
        download_data_file(load_and_validate_config(HfDataConfig, argv=argv))
    else:
        raise SystemExit("usage: hf_download {model|data} [--field=value ...]")


if __name__ == "__main__":
    main()

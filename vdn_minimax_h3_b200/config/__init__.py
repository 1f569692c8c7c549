from vdn_minimax_h3_b200.config.loader import ConfigError, load_config, merge, resolved_dict  # noqa: F401
from vdn_minimax_h3_b200.config.schemas import (InferenceConfig, StageA1Config,  # noqa: F401
                                                StageA2Config, StageBConfig, StageDMDConfig)

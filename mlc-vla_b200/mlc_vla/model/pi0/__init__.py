"""π0.5 model for the B200 build. Importing this package needs neither TVM nor a GPU."""

from .pi0_config import GemmaExpertConfig, Pi0Config, SiglipConfig
from .pi0_model import Pi0Model

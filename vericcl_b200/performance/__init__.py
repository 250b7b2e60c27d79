"""Cost model and exact event simulator (reference layer L1)."""
from .model import CostModel, RateProfile, ServiceCost
from .events import Executable, Movement, WorkOperation
from .simulation import Prediction, predict
from .initial import initial_cost_model, model_context

__all__ = ["CostModel", "RateProfile", "ServiceCost", "Executable", "Movement", "WorkOperation", "Prediction",
           "predict", "initial_cost_model", "model_context"]

"""Training stack (brain-train): Trainer/TrainerBuilder, Batch, callbacks, metrics, ModelState."""
from .trainer import (Batch, SyntheticClassification, TrainStep, TrainingSummary, Trainer, TrainerBuilder,  # noqa: F401
                      L1Regularizer, L2Regularizer, perplexity)
from .callbacks import (TrainingCallback, EarlyStopping, MetricHistoryLogger, JsonlStepLogger, RunningAverage,  # noqa: F401
                        AccuracyMetric, TopKAccuracyMetric, CheckpointMeta, BestModelTracker)
from ..checkpoint.formats import ModelState  # noqa: F401
from .callbacks import (CallbackAction, check_improvement, argmax_rows, WindowedAverage,  # noqa: F401
                        TensorModuleAdapter, TrainableModule)
from .trainer import L2Regularizer as L2Regularization  # noqa: F401  (the reference's name)

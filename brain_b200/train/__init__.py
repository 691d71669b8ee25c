"""Training stack (brain-train): Trainer/TrainerBuilder, Batch, callbacks, metrics, ModelState."""
from .trainer import (Batch, SyntheticClassification, TrainStep, TrainingSummary, Trainer, TrainerBuilder,  # noqa: F401
                      L1Regularizer, L2Regularizer, perplexity)
from .callbacks import (TrainingCallback, EarlyStopping, MetricHistoryLogger, JsonlStepLogger, RunningAverage,  # noqa: F401
                        AccuracyMetric, TopKAccuracyMetric, CheckpointMeta, BestModelTracker)
from ..checkpoint.formats import ModelState  # noqa: F401

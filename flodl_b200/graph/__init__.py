"""Graph builder (FlowBuilder) and executable graphs with graph-tree composition."""
from .control import (ArgmaxSelector, FixedSelector, LearnedHalt, SigmoidRouter,  # noqa: F401
                      SoftmaxRouter, ThresholdHalt)
from .flow import FlowBuilder, MergeOp  # noqa: F401
from .graph import Graph  # noqa: F401
from .trend import Trend, TrendGroup  # noqa: F401

"""Joint sequence x layer CP planning (public API of the reference's ``joint_cp``)."""

from .cost import Evaluator, Model, execution_contract, resource_metrics
from .ir import Group, Layout, Microbatch, Plan, route, spans, validate_layout, validate_plan
from .solver import SearchLimit, SearchOptions, layout_candidates, rank_partitions, solve

__all__ = ["Group", "Layout", "Microbatch", "Plan", "Model", "SearchOptions", "solve", "validate_plan",
           "Evaluator", "SearchLimit", "layout_candidates", "rank_partitions", "route", "spans",
           "validate_layout", "execution_contract", "resource_metrics"]

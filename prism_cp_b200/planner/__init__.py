"""CPU planner: joint 2-D plans, the 1-D planner, native N, capacity policies."""

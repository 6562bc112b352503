"""Data-source classes (importable under the reference's module name for --data-source-path)."""
from miles_b200.rollout.data import (DataSource, RolloutDataSource,  # noqa: F401
                                     RolloutDataSourceWithBuffer, pop_first)

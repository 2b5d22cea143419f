"""Onboarding step 2a: regenerate the rewriter's node handlers from target_node_names.yaml."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from centrifuge_b200.filter.codegen import main  # noqa: E402

if __name__ == "__main__":
    main()

"""Onboarding step 1: probe a model's backward node types into target_node_names.yaml.

    cd grad_filter && python add_torch_native_model.py --model_path <name-or-dir> [--use_lora]
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from centrifuge_b200.filter.probe import main  # noqa: E402

if __name__ == "__main__":
    main()

"""ugdr_b200.ops"""

"""ugdr_b200.utils"""

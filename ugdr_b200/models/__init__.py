"""ugdr_b200.models"""

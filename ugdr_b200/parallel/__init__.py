"""ugdr_b200.parallel"""

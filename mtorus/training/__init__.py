"""mtorus.training"""

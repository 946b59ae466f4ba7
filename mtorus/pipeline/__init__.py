"""mtorus.pipeline"""

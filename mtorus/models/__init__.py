"""mtorus.models"""

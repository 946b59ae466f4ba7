"""mtorus.comm"""

#pragma once
#include "lammps_mock.h"
